"""Pin the CPU oracle to the reference package's own outputs (tests/golden/).

The fixtures were produced by running the reference RefineKV v0.1.2 PyTorch
backend (``tests/golden/make_golden.py``).  The oracle restates the same
algorithm and must reproduce those outputs bit for bit on this CPU.
"""

import pytest
import torch

from helpers import checksum, reference_inputs, sha256
from oracle import refinekv_oracle as ora
from refinekv_b200 import synthetic

SUMMARY_NAMES = ("counts", "key_mean", "value_mean", "ellipsoid", "value_norm", "max_value_norm")


def _assert_summary(summary, expected):
    for name in SUMMARY_NAMES:
        got = getattr(summary, name)
        want = expected[name]
        if isinstance(want, dict):
            assert want["shape"] == tuple(got.shape), name
            assert want["sha256"] == sha256(got), name
        else:
            assert got.dtype == want.dtype, name
            assert torch.equal(got, want), name


def test_fixture_provenance(golden):
    assert golden["reference_version"] == "0.1.2"


def test_summary_cases_bit_exact(golden):
    for case in golden["summary_cases"]:
        s = ora.build_summary(case["keys"], case["values"], case["block"], case["chunk"])
        _assert_summary(s, case["out"])
        assert torch.equal(s.keys, case["key_pages"])
        assert torch.equal(s.values, case["value_pages"])
        assert s.keys.stride()[1:] == (case["block"] * s.keys.shape[-1], s.keys.shape[-1], 1)


def _regenerate(case):
    if case["keys"] is not None:
        return case["q"], case["keys"], case["values"]
    q, keys, values = reference_inputs(case["length"], case["dim"], case["seed"])
    assert [checksum(q), checksum(keys), checksum(values)] == case["input_checksum"]
    return q, keys, values


@pytest.mark.parametrize("index", range(4))
def test_agreement_cases_bit_exact(golden, index):
    case = golden["agreement_cases"][index]
    q, keys, values = _regenerate(case)
    s = ora.build_summary(keys, values, case["block"])
    _assert_summary(s, case["summary"])
    z, risk, log_z, log_c = ora.selection_statistics(q, s)
    for got, name in ((z, "z"), (risk, "risk"), (log_z, "log_z"), (log_c, "log_c")):
        assert torch.equal(got, case[name]), name
    mask, _ = ora.select_blocks(q, s, case["eps"], case["reduction"])
    assert torch.equal(mask, case["mask"])
    for n, rec in case["attention"].items():
        out, sel = ora.sparse_attention(q, s, keys[:, :n], values[:, :n], case["eps"],
                                        case["reduction"], anchor_mask=case["anchor"])
        assert torch.equal(sel, rec["selected"])
        assert torch.equal(out, rec["output"]), n


def test_known_answer(golden):
    case = golden["special_cases"]["known_answer"]
    s = ora.build_summary(case["keys"], case["values"], case["block"])
    out, sel = ora.sparse_attention(case["q"], s, case["keys"][:, :0], case["values"][:, :0],
                                    case["eps"], case["reduction"])
    assert not sel.any()
    assert torch.equal(out, case["output"])
    torch.testing.assert_close(out, torch.full_like(out, (16 + 9) / 19))


def test_large_query_stays_finite(golden):
    case = golden["special_cases"]["large_query"]
    s = ora.build_summary(case["keys"], case["values"], case["block"])
    z, risk, log_z, log_c = ora.selection_statistics(case["q"], s)
    assert torch.equal(risk, case["risk"])
    out, sel = ora.sparse_attention(case["q"], s, case["keys"][:, :0], case["values"][:, :0],
                                    case["eps"], case["reduction"])
    assert torch.equal(sel, case["selected"])
    assert torch.equal(out, case["output"])
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("index", range(2))
def test_synthetic_workload_bit_exact(golden, index):
    case = golden["synthetic_cases"][index]
    dtype = torch.float32 if case["dtype"] == "torch.float32" else torch.bfloat16
    data = synthetic.make_layer(case["seed"], case["layer"], case["heads"], case["tokens"],
                                case["dim"], case["block"], dtype=dtype)
    assert [checksum(data.keys), checksum(data.values)] == case["input_checksum"]
    s = ora.build_summary(data.keys, data.values, case["block"])
    _assert_summary(s, case["summary"])
    anchor_q = synthetic.make_queries(case["seed"], case["layer"], -1, data.planted_mean,
                                      case["group"], case["anchors"], dtype)
    anchor = ora.anchor_union(anchor_q, s, case["eps"], case["reduction"])
    assert torch.equal(anchor, case["anchor_mask"])
    ks, vs = [], []
    for step, rec in enumerate(case["per_step"]):
        k, v = synthetic.make_decode_token(case["seed"], case["layer"], step, case["heads"],
                                           case["dim"], case["tokens"] + step, dtype)
        ks.append(k)
        vs.append(v)
        assert torch.equal(rec["q"], synthetic.make_queries(
            case["seed"], case["layer"], step, data.planted_mean, case["group"], 1, dtype)[0])
        z, risk, _, _ = ora.selection_statistics(rec["q"], s)
        assert torch.equal(risk, rec["risk"])
        out, sel = ora.sparse_attention(rec["q"], s, torch.cat(ks, 1), torch.cat(vs, 1),
                                        case["eps"], case["reduction"], anchor_mask=anchor)
        assert torch.equal(sel, rec["selected"])
        assert torch.equal(out, rec["output"])


def test_margin_classifier_and_merge():
    q, keys, values = reference_inputs(71, 64)
    s = ora.build_summary(keys, values, 16)
    _, risk, _, _ = ora.selection_statistics(q, s)
    eps = float(risk[0, 0, 2])
    margin = ora.margin_blocks(q, s, eps, "any")
    assert margin[0, 2]
    assert not ora.margin_blocks(q, s, 1e9, "any").any()
    # the split merge of two halves equals one softmax
    logits = torch.randn(3, 10)
    vals = torch.randn(10, 8)
    full = logits.softmax(-1) @ vals
    parts = []
    for sl in (slice(0, 4), slice(4, 10)):
        m = logits[:, sl].amax(-1)
        p = (logits[:, sl] - m[:, None]).exp()
        parts.append((m, p.sum(-1), p @ vals[sl]))
    m = torch.stack([p[0] for p in parts], -1)
    l = torch.stack([p[1] for p in parts], -1)
    o = torch.stack([p[2] for p in parts], -2)
    torch.testing.assert_close(ora.merge_partials(m, l, o), full)

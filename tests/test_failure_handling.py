"""Failure handling without faulting a GPU.

* Device: every kernel's mbarrier wait is bounded and reports a timeout in
  the workspace status word instead of hanging.  `rkv_selftest_wait_timeout`
  runs that exact wait on an mbarrier nothing completes, with a short limit;
  the test checks the status bit and that the context keeps working.
* Host, multi-rank: a rank that leaves before an exchange must not hang the
  others: with a short process-group timeout the surviving rank's next
  collective ends with an error (gloo ranks on the CPU; the NCCL path uses the
  same helper and `SplitDecode` passes the caller's group, whose timeout
  applies the same way).
"""

from __future__ import annotations

import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from refinekv_b200 import RefineKVConfig, _native, build_summary, parallel, sparse_attention, synthetic
from refinekv_b200.attention import device_status


def test_selftest_rejects_bad_arguments_without_a_device():
    lib = _native.load()
    assert lib.rkv_selftest_wait_timeout(None, 1000, None) == _native.RKV_ERR_INVALID_ARGUMENT
    assert b"status" in lib.rkv_last_error()


@pytest.mark.gpu
def test_bounded_wait_reports_timeout_and_the_context_survives():
    lib = _native.load()
    status = torch.zeros(1, device="cuda", dtype=torch.int32)
    t0 = time.perf_counter()
    _native.check(lib.rkv_selftest_wait_timeout(status.data_ptr(), 2_000_000,
                                                torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert int(status.item()) == _native.DEVICE_TIMEOUT
    # the same context still runs the decode path and its status stays clean
    data = synthetic.make_layer(3, 0, 2, 2048, 128, 32, device="cuda")
    cfg = RefineKVConfig(eps=0.01)
    s = build_summary(data.keys, data.values, cfg)
    q = synthetic.make_queries(3, 0, 0, data.planted_mean, 4)[0]
    ws = {}
    out = sparse_attention(q, s, data.keys[:, :5].contiguous(), data.values[:, :5].contiguous(),
                           cfg, workspace=ws).output
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert device_status(ws) == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _leaving_rank(rank, world, port, results):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=3))
    slab = 16
    buf = torch.zeros(world * slab, dtype=torch.uint8)
    buf[rank * slab:(rank + 1) * slab] = rank + 1
    parallel.all_gather_slabs(buf, slab, rank, None)  # one good step
    if rank == world - 1:
        results[rank] = "left"
        os._exit(0)  # leaves between steps, with nothing in flight
    t0 = time.monotonic()
    try:
        parallel.all_gather_slabs(buf, slab, rank, None)
        results[rank] = "no error"
    except Exception as error:  # the collective must end, not hang
        results[rank] = f"error after {time.monotonic() - t0:.1f}s: {type(error).__name__}"


def test_gloo_rank_leaving_ends_the_survivors_collective_with_an_error():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_leaving_rank, args=(r, 2, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=60)
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join()
                pytest.fail("a rank hung instead of ending with an error")
        assert results.get(1) == "left"
        assert str(results.get(0, "")).startswith("error after"), dict(results)

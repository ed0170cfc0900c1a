"""The embedding gather's NCCL entry points on the GPU: correct in rank order,
and bounded when a peer is missing. Every rank runs in a spawned child
process (NVLS off, as on this pool a rank that dies while bound to an NVLink
multicast object faults its peers); the parent only reads what each child
recorded, so a child that fails or stalls cannot take the test runner with it.

  * one GPU: a rank whose peer never joins gives up at its deadline (the
    communicator is aborted during its rendezvous, ERR_TIMEOUT) and the
    context still runs kernels afterwards;
  * two GPUs: two ranks gather each other's embeddings in rank order; then
    one rank leaves between steps (its stream drained, nothing in flight) and
    the other's next gather ends in ERR_TIMEOUT or ERR_COMM within its
    deadline, after which its context still runs kernels.
"""
from __future__ import annotations

import json
import multiprocessing
import os
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _file_exchange(path, rank):
    def exchange(mine):
        if rank == 0:
            with open(path + ".tmp", "wb") as f:
                f.write(mine)
            os.replace(path + ".tmp", path)
            return mine
        t_end = time.monotonic() + 60
        while not os.path.exists(path):
            if time.monotonic() > t_end:
                raise TimeoutError("no rendezvous id")
            time.sleep(0.05)
        with open(path, "rb") as f:
            return f.read()
    return exchange


def _scale_still_runs():
    import torch

    from hexlib_b200 import _lib
    x = torch.arange(1024, dtype=torch.float16, device="cuda")
    y = torch.empty_like(x)
    rc = _lib.lib().hexlib_b200_scale_fp16(x.data_ptr(), y.data_ptr(), 1024, 2.0,
                                           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc == 1 and bool(torch.equal(y, x * 2))


def _lonely_rank(out_dir):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    from hexlib_b200 import dist as D
    torch.cuda.set_device(0)
    rec = {}
    t0 = time.monotonic()
    try:
        D.EmbeddingGather(0, 2, 0, timeout_s=3.0,
                          exchange=_file_exchange(os.path.join(out_dir, "id"), 0))
        rec["status"] = 1
    except D.CommError as e:
        rec["status"] = e.status
    rec["seconds"] = time.monotonic() - t0
    rec["kernels_run"] = _scale_still_runs()
    with open(os.path.join(out_dir, "lonely.json"), "w") as f:
        json.dump(rec, f)
    os._exit(0)       # the aborted communicator has nothing left to release


def test_a_peer_that_never_joins_times_out_and_the_context_survives(tmp_path):
    from hexlib_b200 import _lib, wire
    if not _lib.lib().hexlib_b200_nccl_available():
        pytest.skip("NCCL cannot be loaded")
    ctx = multiprocessing.get_context("spawn")
    p = ctx.Process(target=_lonely_rank, args=(str(tmp_path),))
    p.start()
    p.join(timeout=120)
    if p.is_alive():
        p.kill()
        p.join()
    rec = json.loads((tmp_path / "lonely.json").read_text())
    assert rec["status"] == wire.STATUS["ERR_TIMEOUT"], rec
    assert 2.5 < rec["seconds"] < 30, rec
    assert rec["kernels_run"]


def _pair_rank(rank, out_dir):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    from hexlib_b200 import dist as D
    torch.cuda.set_device(rank)
    rec = {"rank": rank}
    stream = torch.cuda.current_stream().cuda_stream
    g = D.EmbeddingGather(rank, 2, rank, timeout_s=5.0,
                          exchange=_file_exchange(os.path.join(out_dir, "id"), rank))
    local = (torch.arange(2 * 8 * 16, dtype=torch.float32, device="cuda").reshape(2, 8, 16)
             + 1000 * rank).to(torch.float16)
    full = torch.empty((4, 8, 16), dtype=torch.float16, device="cuda")
    g.gather(local, full, stream)
    g.wait(stream)
    np.save(os.path.join(out_dir, f"full{rank}.npy"), full.cpu().numpy())
    torch.cuda.synchronize()
    if rank == 1:             # leaves between steps: nothing of it is in flight
        open(os.path.join(out_dir, "left"), "w").close()
        os._exit(0)
    t_end = time.monotonic() + 30
    while not os.path.exists(os.path.join(out_dir, "left")) and time.monotonic() < t_end:
        time.sleep(0.05)
    time.sleep(0.5)
    t0 = time.monotonic()
    try:
        g.gather(local, full, stream)
        g.wait(stream)
        rec["status"] = 1
    except D.CommError as e:
        rec["status"] = e.status
    rec["seconds"] = time.monotonic() - t0
    rec["kernels_run"] = _scale_still_runs()
    with open(os.path.join(out_dir, "rank0.json"), "w") as f:
        json.dump(rec, f)
    os._exit(0)


def test_two_ranks_gather_in_rank_order_and_a_rank_that_leaves_is_bounded(tmp_path):
    import torch

    from hexlib_b200 import _lib, wire
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    if not _lib.lib().hexlib_b200_nccl_available():
        pytest.skip("NCCL cannot be loaded")
    ctx = multiprocessing.get_context("spawn")
    procs = [ctx.Process(target=_pair_rank, args=(r, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    want = np.concatenate([(np.arange(256, dtype=np.float32).reshape(2, 8, 16) + 1000 * r)
                           .astype(np.float16) for r in range(2)])
    for r in range(2):
        np.testing.assert_array_equal(np.load(tmp_path / f"full{r}.npy"), want)
    rec = json.loads((tmp_path / "rank0.json").read_text())
    assert rec["status"] in (wire.STATUS["ERR_TIMEOUT"], wire.STATUS["ERR_COMM"]), rec
    assert rec["seconds"] < 30, rec
    assert rec["kernels_run"]

"""The multi-GPU host logic on CPU ranks: two `gloo` processes shard a batch by
image, each produces its shard's embeddings, and the all-gather hands every
rank the whole batch in rank order. A rank that fails is seen by the other as
an error from its next collective, within the process group's timeout."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hexlib_b200 import dist as D


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir, fail_rank):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=20))
    r, lr, w = D.env_rank()
    sh = D.shard(8, r, w)
    # stand-in embeddings: each image's rows carry its global image index
    local = torch.arange(sh.start, sh.start + sh.count, dtype=torch.float16)
    local = local[:, None, None].expand(sh.count, 4, 3).contiguous()
    if rank == fail_rank:
        raise SystemExit(3)       # leaves before the collective
    try:
        full = D.gather_embeddings(local)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), full.numpy())
    except Exception as e:  # noqa: BLE001 -- recorded for the parent
        with open(os.path.join(out_dir, f"rank{rank}.err"), "w") as f:
            f.write(type(e).__name__)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def test_shard_arithmetic():
    assert [D.shard(64, r, 8) for r in (0, 7)] == [D.Shard(0, 8, 0, 8), D.Shard(7, 8, 56, 8)]
    with pytest.raises(ValueError):
        D.shard(10, 0, 4)
    with pytest.raises(ValueError):
        D.shard(8, 2, 2)


def test_two_gloo_ranks_gather_the_whole_batch(tmp_path):
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path), -1), nprocs=2,
                       start_method="spawn", join=True)
    for rank in range(2):
        full = np.load(tmp_path / f"rank{rank}.npy")
        assert full.shape == (8, 4, 3)
        np.testing.assert_array_equal(full[:, 0, 0], np.arange(8, dtype=np.float16))


def test_a_rank_that_leaves_is_an_error_for_the_other(tmp_path):
    import multiprocessing
    port = _free_port()
    ctx = multiprocessing.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path), 1)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    for p in procs:
        if p.is_alive():          # never expected: the group timeout is 20 s
            p.kill()
            p.join()
    assert procs[1].exitcode == 3
    assert not (tmp_path / "rank0.npy").exists()
    assert (tmp_path / "rank0.err").exists()

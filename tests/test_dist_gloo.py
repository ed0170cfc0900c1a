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


def _id_worker(rank, world, port, out_dir, leave_rank):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=20))
    if rank == leave_rank:
        raise SystemExit(3)       # leaves before the rendezvous id is shared
    try:
        ident = D.share_unique_id(rank)
        with open(os.path.join(out_dir, f"id{rank}.bin"), "wb") as f:
            f.write(ident)
    except Exception as e:  # noqa: BLE001 -- recorded for the parent
        with open(os.path.join(out_dir, f"id{rank}.err"), "w") as f:
            f.write(type(e).__name__)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def test_every_rank_receives_rank0s_nccl_rendezvous_id(tmp_path):
    """The id is made by the library (no GPU needed) on rank 0 only and
    reaches every rank byte for byte through the process group."""
    from hexlib_b200 import _lib
    if not _lib.lib().hexlib_b200_nccl_available():
        pytest.skip("NCCL cannot be loaded in this process")
    port = _free_port()
    mp.start_processes(_id_worker, args=(3, port, str(tmp_path), -1), nprocs=3,
                       start_method="spawn", join=True)
    ids = [(tmp_path / f"id{r}.bin").read_bytes() for r in range(3)]
    assert len(ids[0]) == 128 and ids[0] == ids[1] == ids[2] and any(ids[0])


def test_a_rank_that_leaves_before_the_rendezvous_is_an_error_for_the_others(tmp_path):
    import multiprocessing
    port = _free_port()
    ctx = multiprocessing.get_context("spawn")
    procs = [ctx.Process(target=_id_worker, args=(r, 2, port, str(tmp_path), 1))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    for p in procs:
        if p.is_alive():          # never expected: the group timeout is 20 s
            p.kill()
            p.join()
    assert procs[1].exitcode == 3
    assert not (tmp_path / "id0.bin").exists()
    assert (tmp_path / "id0.err").exists()


def test_the_nccl_entries_refuse_bad_arguments_without_a_device():
    import ctypes

    from hexlib_b200 import _lib, wire
    L = _lib.lib()
    h = ctypes.c_void_p()
    ident = (ctypes.c_uint8 * 128)()
    for nranks, rank, timeout in ((0, 0, 100), (2, 2, 100), (2, -1, 100), (2, 0, 0)):
        assert L.hexlib_b200_nccl_open(ident, nranks, rank, 0, timeout, ctypes.byref(h)) == \
            wire.STATUS["ERR_INVAL_PARAMS"]
        assert h.value is None
    assert L.hexlib_b200_nccl_allgather_f16(None, None, None, 8, None, 100) == \
        wire.STATUS["ERR_NOT_STARTED"]
    assert L.hexlib_b200_nccl_wait(None, None, 100) == wire.STATUS["ERR_NOT_STARTED"]
    assert L.hexlib_b200_nccl_unique_id(None) == wire.STATUS["ERR_INVAL_PARAMS"]
    assert L.hexlib_b200_nccl_close(None, 0) == wire.STATUS["OK"]


def test_the_gather_refuses_tensors_off_its_device_before_calling_nccl():
    import pytest
    import torch

    from hexlib_b200 import dist as D
    g = object.__new__(D.EmbeddingGather)     # no communicator: the checks come first
    g.rank, g.world, g.device, g.timeout_ms, g._h = 0, 2, 0, 100, None
    local = torch.zeros((2, 4), dtype=torch.float16)
    out = torch.zeros((4, 4), dtype=torch.float16)
    with pytest.raises(ValueError, match="cuda:0"):
        g.gather(local, out, 0)
    with pytest.raises(TypeError):
        g.gather(local.float(), out, 0)
    with pytest.raises(ValueError, match="world x local"):
        g.gather(local, out[:3], 0)

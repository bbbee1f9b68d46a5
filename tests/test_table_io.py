"""On-disk format of the row-sharded table (host_pool.py:90-108 layout,
:175-188 snapshots): a world-size-4 gloo save of a strided table, reloaded
at world sizes 1, 2 and 3; float16 values; the reference's own readers
(np.load of <key>.npy, shapes and dtypes of a live pool) see the same
arrays.  CPU tensors; the device path is covered in test_table_io_gpu.py."""

import os
import socket

import numpy as np
import pytest
import torch

from model_b200.table_io import load_table, open_table, save_table


def _table(n, d, dtype=np.float32, seed=0):
    rng = np.random.default_rng(seed)
    return {"values": rng.standard_normal((n, d)).astype(dtype), "acc": rng.random(n).astype(np.float32),
            "m": rng.standard_normal((n, d)).astype(np.float32), "v": rng.random((n, d)).astype(np.float32)}


def test_single_rank_round_trip_and_reference_reader(tmp_path):
    full = _table(1000, 16)
    save_table(str(tmp_path), {k: torch.from_numpy(a) for k, a in full.items()}, 1000)
    for k, a in full.items():
        np.testing.assert_array_equal(np.load(tmp_path / f"{k}.npy"), a)     # what HostPool.load reads
    assert not any(p.name.endswith(".tmp.npy") for p in tmp_path.iterdir())
    got = load_table(str(tmp_path), ["values", "acc", "m", "v"])
    for k, a in full.items():
        np.testing.assert_array_equal(got[k].numpy(), a)


@pytest.mark.parametrize("world", [2, 3, 8])
def test_load_any_world_size(tmp_path, world):
    full = _table(77, 8, np.float16, seed=world)
    save_table(str(tmp_path), {"values": torch.from_numpy(full["values"]), "acc": torch.from_numpy(full["acc"])}, 77)
    rows = 0
    for r in range(world):
        got = load_table(str(tmp_path), ["values", "acc", "m"], rank=r, world=world)
        assert "m" not in got                                   # missing files are skipped
        assert got["values"].dtype == torch.float16
        np.testing.assert_array_equal(got["values"].numpy(), full["values"][r::world])
        np.testing.assert_array_equal(got["acc"].numpy(), full["acc"][r::world])
        rows += got["values"].shape[0]
    assert rows == 77
    as32 = load_table(str(tmp_path), ["values"], dtype=torch.float32)["values"]
    np.testing.assert_array_equal(as32.numpy(), full["values"].astype(np.float32))


def test_save_rejects_wrong_local_rows(tmp_path):
    with pytest.raises(ValueError):
        save_table(str(tmp_path), {"values": torch.zeros(10, 4)}, 100, rank=1, world=4)
    with pytest.raises(ValueError):
        save_table(str(tmp_path), {"acc": torch.zeros(25, 2)}, 100, rank=0, world=4)
    with pytest.raises(ValueError):
        save_table(str(tmp_path), {"weights": torch.zeros(25, 2)}, 100, rank=0, world=4)


def test_open_table_matches_reference_layout(tmp_path):
    arrs = open_table(str(tmp_path), 600, 8, np.float16, optimizer="rowwise_adagrad", seed=3)
    assert set(arrs) == {"values", "acc"}
    assert arrs["values"].shape == (600, 8) and arrs["values"].dtype == np.float16
    assert arrs["acc"].shape == (600,) and not arrs["acc"].any()
    want = (np.random.default_rng(3).standard_normal((600, 8)) * 8 ** -0.5).astype(np.float16)
    np.testing.assert_array_equal(np.asarray(arrs["values"]), want)
    arrs["values"][5] = 1.0
    arrs["values"].flush()
    again = open_table(str(tmp_path), 600, 8, np.float16, optimizer="rowwise_adagrad")
    assert (np.asarray(again["values"][5]) == 1.0).all()                 # reopened, not re-initialised
    with pytest.raises(ValueError):
        open_table(str(tmp_path), 601, 8, np.float16)
    adam = open_table(str(tmp_path / "adam"), 10, 4, optimizer="adam")
    assert set(adam) == {"values", "m", "v"}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, dest):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = _table(1003, 12, seed=11)
        local = {k: torch.from_numpy(np.ascontiguousarray(a[rank::world])) for k, a in full.items()}
        save_table(dest, local, 1003, rank=rank, world=world)
    finally:
        dist.destroy_process_group()


def test_gloo_four_ranks_save_then_reshard(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(4, _free_port(), str(tmp_path)), nprocs=4, join=True)
    full = _table(1003, 12, seed=11)
    for k, a in full.items():
        np.testing.assert_array_equal(np.load(tmp_path / f"{k}.npy"), a)
    for world in (1, 2, 3):
        for r in range(world):
            got = load_table(str(tmp_path), ["values", "acc"], rank=r, world=world)
            np.testing.assert_array_equal(got["values"].numpy(), full["values"][r::world])
            np.testing.assert_array_equal(got["acc"].numpy(), full["acc"][r::world])


def _bad_rank_worker(rank, world, port, dest, outdir):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        full = _table(101, 4, seed=2)
        local = {"values": torch.from_numpy(np.ascontiguousarray(full["values"][rank::world]))}
        if rank == 1:
            local["values"] = local["values"][:-1]                       # one row short
        msg = ""
        try:
            save_table(dest, local, 101, rank=rank, world=world)
        except ValueError as e:
            msg = str(e)
        with open(os.path.join(outdir, f"bad{rank}.txt"), "w") as f:
            f.write(msg)
    finally:
        dist.destroy_process_group()


def test_gloo_bad_rows_on_one_rank_fail_every_rank(tmp_path):
    """A rank with wrong arguments makes every rank raise before the first
    barrier, instead of leaving the others blocked in a collective."""
    import torch.multiprocessing as mp
    dest = tmp_path / "snap"
    mp.spawn(_bad_rank_worker, args=(3, _free_port(), str(dest), str(tmp_path)), nprocs=3, join=True)
    for r in range(3):
        msg = (tmp_path / f"bad{r}.txt").read_text()
        assert "rank 1:" in msg and "local rows" in msg, (r, msg)
    assert not (dest / "values.npy").exists()

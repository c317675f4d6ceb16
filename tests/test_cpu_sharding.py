"""Host logic of the row-sharded decode on CPU: the row partition and the
all-gather assembly of per-rank list slices (gloo, world size 2)."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import torch_dbs_extension as ext


@pytest.mark.parametrize("rows,world", [(1, 1), (7, 2), (8, 2), (100, 3), (5, 8), (4096, 8)])
def test_row_shards_cover_every_row_once(rows, world):
    per, ranges = ext.row_shards(rows, world)
    assert len(ranges) == world
    seen = []
    for r, (b, e) in enumerate(ranges):
        assert b == min(rows, r * per) and b <= e <= b + per
        seen.extend(range(b, e))
    assert seen == list(range(rows))


def _gather_worker(rank, world, port, path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rows, C = 11, 3
        per, ranges = ext.row_shards(rows, world)
        lists = torch.full((world * per, C), -1, dtype=torch.int64)
        b, e = ranges[rank]
        for r in range(b, e):   # what this rank's scan writes: its own rows only
            lists[r] = torch.arange(C) + 100 * r
        out = [torch.empty((per, C), dtype=torch.int64) for _ in range(world)]
        dist.all_gather(out, lists[rank * per:(rank + 1) * per].clone())
        full = torch.cat(out)
        ok = all(torch.equal(full[r], torch.arange(C) + 100 * r) for r in range(rows))
        if rank == 0:
            with open(path, "w") as f:
                f.write("ok" if ok else "bad")
    finally:
        dist.destroy_process_group()


def test_list_slices_assemble_over_gloo(tmp_path):
    path = tmp_path / "r.txt"
    mp.start_processes(_gather_worker, args=(2, 29623, str(path)), nprocs=2, start_method="spawn")
    assert path.read_text() == "ok"

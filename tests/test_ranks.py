"""Windows across ranks (whispereacp_b200/ranks.py): the split, the
max-over-ranks time and the gather, as two gloo ranks on the CPU."""
import os
import socket

import numpy as np
import pytest

from whispereacp_b200.ranks import window_range


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_window_ranges_partition_the_batch(world):
    for total in range(0, 21):
        ranges = [window_range(total, r, world) for r in range(world)]
        assert [w for r in ranges for w in r] == list(range(total))
        sizes = [len(r) for r in ranges]
        assert max(sizes) - min(sizes) <= 1


def test_window_range_refuses_a_rank_outside_the_world():
    with pytest.raises(ValueError):
        window_range(8, 2, 2)
    with pytest.raises(ValueError):
        window_range(-1, 0, 1)


class _FakeDecoder:
    """Stands in for a Decoder on a CPU rank: each window's "transcript" is
    derived from its own encoder rows, so order mistakes show."""

    def __init__(self, windows):
        self.windows = windows
        self.closed = False

    def transcribe(self, rows, cross_positions=0):
        assert rows.shape[0] == self.windows
        return [np.array([int(r[0, 0]), int(r[0, 0]) + 1000], dtype=np.uint32) for r in rows]

    def close(self):
        self.closed = True


def _rank_main(rank, world, port, total, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    from whispereacp_b200 import ranks
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        worst = ranks.max_over_ranks([rank + 1.5, 10.0 - rank])
        rows = np.zeros((total, 3, 4), np.float32)
        rows[:, 0, 0] = np.arange(total) * 7
        gathered = ranks.transcribe_windows(_FakeDecoder, rows)
        np.save(os.path.join(out_dir, f"max{rank}.npy"), np.array(worst))
        if rank == 0:
            np.save(os.path.join(out_dir, "gathered.npy"), np.stack(gathered) if gathered else np.zeros((0, 2)))
        else:
            assert gathered is None
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("total", [5, 1])
def test_two_gloo_ranks_split_time_and_gather(tmp_path, total):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), total, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    for rank in range(world):
        assert np.load(tmp_path / f"max{rank}.npy").tolist() == [2.5, 10.0]
    gathered = np.load(tmp_path / "gathered.npy")
    assert gathered.shape == (total, 2)
    assert gathered[:, 0].tolist() == [7 * w for w in range(total)]

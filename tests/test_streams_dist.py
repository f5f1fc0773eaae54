"""Multi-stream sharding and the final chunk gather, as world_size-2 gloo
ranks on CPU (the host logic of the multi-GPU bench path)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from reflex_b200.streams import gather_chunks, shard_range


@pytest.mark.parametrize("n,world", [(64, 8), (5, 2), (7, 3), (1, 1), (9, 4)])
def test_shard_range_covers_every_stream_once(n, world):
    seen = []
    for r in range(world):
        s, c = shard_range(n, r, world)
        seen += list(range(s, s + c))
    assert seen == list(range(n))


def test_shard_range_rejects_bad_input():
    with pytest.raises(ValueError):
        shard_range(0, 0, 1)
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_streams, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s, c = shard_range(n_streams, rank, world)
        # each stream's "action chunk" is filled with its global stream id
        local = torch.arange(s, s + c, dtype=torch.float32).view(c, 1, 1).expand(c, 50, 32).contiguous()
        out = gather_chunks(local, n_streams, dist)
        q.put((rank, out[:, 0, 0].tolist(), tuple(out.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_streams", [5, 8])
def test_gather_chunks_two_ranks(n_streams):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_streams, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ids, shape in res:
        assert shape == (n_streams, 50, 32)
        assert ids == [float(i) for i in range(n_streams)]

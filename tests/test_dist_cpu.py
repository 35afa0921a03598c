"""Host-side logic of the tensor-parallel communicator on CPU ranks (gloo)."""
import socket

import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port):
    import datetime
    import torch.distributed as dist
    from python.kinetic_rt.dist import exchange_handles
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        got = exchange_handles(bytes([rank]) * 64)
        assert got == [bytes([r]) * 64 for r in range(world)]
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_handle_exchange_rank_order(world):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(world, _free_port()), nprocs=world, join=True)

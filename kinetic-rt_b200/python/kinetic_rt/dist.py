"""Tensor-parallel communicator over NVLink peer buffers.

One process per GPU.  `TPComm` creates this rank's symmetric buffer in
libkrt (krt_comm_create), exchanges CUDA IPC handles through an initialised
torch.distributed process group (all_gather_object over gloo or NCCL), and
maps the peers' buffers (krt_comm_open_peers).  It then runs the fused
row-parallel GEMM + allreduce and the standalone allreduce; torch.distributed
carries no tensor traffic.
"""
from . import _lib


def exchange_handles(handle, group=None):
    """All-gather one bytes object per rank, returned in rank order."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


class TPComm:
    def __init__(self, rank, world_size, max_n_out, group=None):
        self.rank, self.world_size = int(rank), int(world_size)
        self.has_nccl, self.nccl_threshold = False, None
        self.handle = _lib.comm_create(self.rank, self.world_size, max_n_out)
        if self.world_size > 1:
            mine = _lib.comm_ipc_handle(self.handle)
            _lib.comm_open_peers(self.handle, exchange_handles(mine, group))

    def gemm_ar(self, x, weight, y, workspace, stream=None):
        """y = allreduce_sum(x @ weight^T) across ranks (bf16 tensors on this GPU)."""
        _lib.rowparallel_gemm_ar(self.handle, _lib.gemm_ar_args(x, weight, y, workspace), stream)

    def allreduce(self, send, recv, status, stream=None):
        _lib.allreduce(self.handle, send, recv, status, stream)

    def attach_nccl(self, threshold_bytes, group=None):
        """An NCCL communicator beside the peer buffers (rank 0 makes the id,
        every rank joins); messages of at least threshold_bytes use it."""
        import torch.distributed as dist
        nid = _lib.nccl_unique_id() if self.rank == 0 else None
        ids = [None] * dist.get_world_size(group)
        dist.all_gather_object(ids, nid, group=group)
        _lib.comm_attach_nccl(self.handle, ids[0], threshold_bytes)
        self.has_nccl, self.nccl_threshold = True, int(threshold_bytes)

    def set_nccl_threshold(self, threshold_bytes):
        """Changes the threshold of an attached NCCL communicator (every rank
        must use the same value)."""
        _lib.comm_attach_nccl(self.handle, b"\0" * 128, min(int(threshold_bytes), (1 << 64) - 1))

    def reset(self, group=None, stream=None):
        """Re-agree the exchange state after a peer wait ran out (status bit
        16): every rank drains its stream, zeroes its exchange areas
        (krt_comm_reset) and meets the others at a barrier."""
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier(group=group)  # no rank's kernel still writes into a peer's buffer
        _lib.comm_reset(self.handle, stream)
        dist.barrier(group=group)  # no rank starts a collective before every buffer is clear

    def close(self):
        if self.handle:
            _lib.comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

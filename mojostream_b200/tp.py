"""Host plumbing of tensor parallelism: hand rank 0's group id to every rank.

The library's collectives are NCCL calls made inside libmojostream_cuda.so
(ms_tp_init); the host only has to move one opaque id from rank 0 to the
others before it.  Any transport will do; here torch.distributed (already
initialised, any backend) broadcasts it as bytes.
"""
import torch
import torch.distributed as dist


def broadcast_id(make_id, group=None):
    """Rank 0 calls make_id() (bytes); every rank returns those bytes."""
    rank = dist.get_rank(group)
    backend = dist.get_backend(group)
    device = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else "cpu"
    n = torch.zeros(1, dtype=torch.int64, device=device)
    payload = make_id() if rank == 0 else b""
    if rank == 0:
        n[0] = len(payload)
    dist.broadcast(n, 0, group=group)
    buf = torch.zeros(int(n.item()), dtype=torch.uint8, device=device)
    if rank == 0:
        buf.copy_(torch.frombuffer(bytearray(payload), dtype=torch.uint8))
    dist.broadcast(buf, 0, group=group)
    return bytes(buf.cpu().numpy().tobytes())


def tp_setup(ctx, group=None):
    """ms_tp_init on every rank of the (initialised) process group."""
    from .runtime import tp_unique_id
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    uid = broadcast_id(tp_unique_id, group)
    ctx.tp_init(world, rank, uid)
    return world, rank

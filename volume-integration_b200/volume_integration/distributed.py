"""Training on several GPUs by sharding the views of one scene.

The reference renders one camera per call on one GPU and has no multi-GPU code.
Rendering is independent per view, so the natural split is by camera: one
process per GPU, every rank holds a full replica of the scene parameters
(centres, confidence grids, feature table, linear layer), renders and
back-propagates its own cameras, and the ranks then sum their gradients with
one all-reduce per gradient tensor.  That is the only exchange in a step; with
NCCL over NVLink/NVSwitch it moves 4 bytes per parameter each way.

    shard = views_for_rank(len(cameras), rank, world)
    for v in shard:
        loss(render(cameras[v])).backward()          # gradients accumulate locally
    allreduce_gradients([p.grad for p in params])    # sum over ranks, in place
"""
import torch
import torch.distributed as dist

__all__ = ["views_for_rank", "allreduce_gradients"]


def views_for_rank(n_views, rank, world):
    """Camera indices rank `rank` of `world` renders: round-robin, so shard sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return list(range(rank, n_views, world))


_FLAT = {}


def allreduce_gradients(grads, group=None, coalesce=False):
    """Sums each gradient tensor over the ranks of `group`, in place, and returns them.

    All-reduces are issued asynchronously, largest tensor first (the feature
    table's gradient, then the confidences'), and waited for together, so the
    collectives queue back to back on the communicator's stream.  With
    `coalesce` the gradients are instead copied into one flat buffer (kept for
    the next call of the same size), reduced with a single all-reduce and
    copied back.  `None` entries (parameters without a gradient) are passed
    through; every rank must pass the same shapes in the same order.  With one
    rank this is a no-op.
    """
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return list(grads)
    live = [g for g in grads if g is not None]
    if coalesce and len(live) > 1 and len({(g.device, g.dtype) for g in live}) == 1:
        n = sum(g.numel() for g in live)
        key = (live[0].device, live[0].dtype, n)
        flat = _FLAT.get(key)
        if flat is None:
            flat = _FLAT.setdefault(key, torch.empty(n, dtype=live[0].dtype, device=live[0].device))
        torch.cat([g.reshape(-1) for g in live], out=flat)
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        off = 0
        for g in live:
            g.copy_(flat[off:off + g.numel()].view_as(g))
            off += g.numel()
        return list(grads)
    order = sorted((i for i, g in enumerate(grads) if g is not None), key=lambda i: -grads[i].numel())
    works = []
    for i in order:
        g = grads[i]
        if not g.is_contiguous():
            raise ValueError("allreduce_gradients: gradient tensors must be contiguous")
        works.append(dist.all_reduce(g, op=dist.ReduceOp.SUM, group=group, async_op=True))
    for w in works:
        w.wait()
    return list(grads)

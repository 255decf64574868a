"""View sharding across ranks: the summed gradient of a sharded step equals the
sum of the per-view gradients computed one after another in one process.

* CPU (gloo, world size 2): every rank computes its views' gradients with the
  oracle and calls `allreduce_gradients`; rank 0 compares with the sequential
  sum (fp32 summation order differs: rel 1e-6).
* GPU (NCCL, world size 2, needs two GPUs): the same with the CUDA renderer
  through the autograd Function; compared with the 1-GPU sequential sum within
  the gradient tolerance of the parity tests (atomic order differs).
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for _p in (os.path.join(ROOT, "volume-integration_b200"), os.path.join(ROOT, "oracle"), HERE):
    if _p not in sys.path:
        sys.path.insert(0, _p)

N_VIEWS = 4
GRAD_KEYS = ("dL_dconfidences", "dL_dfeature_table", "dL_dlinear_weights", "dL_dlinear_bias")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _views(device):
    import vi_workloads as wl
    import vi_testlib as tl
    means, conf, kw, _ = wl.make("tiny", table_range=1.0, width=64, height=48, P=1500)
    c = wl.CONFIGS["tiny"]
    cams = wl.orbit(N_VIEWS, c["dist"], 64, 48, c["fov"])
    out = []
    for v, cam in enumerate(cams):
        s = tl.settings_from(kw, cam, device)
        dc, df = tl.random_grads(s, seed=100 + v, device=device)
        out.append((means.to(device), conf.to(device), s, dc, df))
    return out


def _oracle_grads(view):
    import vi_testlib as tl
    means, conf, s, dc, df = view
    _, f = tl.oracle_run(means, conf, s, dc, df)
    return [torch.from_numpy(np.ascontiguousarray(f["grads"][k]).reshape(-1).copy()) for k in GRAD_KEYS]


def _cuda_grads(view):
    import volume_integration as vi
    means, conf, s, dc, df = view
    leaves = [conf.clone().requires_grad_(True), s.feature_table.clone().requires_grad_(True),
              s.linear_weights.clone().requires_grad_(True), s.linear_bias.clone().requires_grad_(True)]
    oc, of, _ = vi.integrate_primitives(means, *leaves, s)
    return [g.reshape(-1).contiguous() for g in torch.autograd.grad([oc, of], leaves, [dc, df])]


def _sharded_sum(rank, world, device, grads_fn):
    from volume_integration.distributed import allreduce_gradients, views_for_rank
    views = _views(device)
    acc = None
    for v in views_for_rank(N_VIEWS, rank, world):
        g = grads_fn(views[v])
        acc = g if acc is None else [a + b for a, b in zip(acc, g)]
    return allreduce_gradients(acc)


def _worker(rank, world, port, backend, out_path):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    if backend == "nccl":
        torch.cuda.set_device(rank)
        device = torch.device("cuda", rank)
        fn = _cuda_grads
    else:
        device = torch.device("cpu")
        fn = _oracle_grads
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        summed = _sharded_sum(rank, world, device, fn)
        if rank == 0:
            torch.save([g.cpu() for g in summed], out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(backend, tmp_path):
    out = str(tmp_path / f"sharded_{backend}.pt")
    mp.start_processes(_worker, args=(2, _free_port(), backend, out), nprocs=2, join=True, start_method="spawn")
    return torch.load(out)


def test_views_for_rank_partitions_the_views():
    from volume_integration.distributed import views_for_rank
    for n in (0, 1, 5, 32):
        for world in (1, 2, 3, 8):
            shards = [views_for_rank(n, r, world) for r in range(world)]
            assert sorted(sum(shards, [])) == list(range(n))
            assert max(map(len, shards)) - min(map(len, shards)) <= 1
    with pytest.raises(ValueError):
        views_for_rank(4, 2, 2)


def test_sharded_gradient_sum_gloo(tmp_path):
    summed = _run("gloo", tmp_path)
    views = _views(torch.device("cpu"))
    seq = None
    for v in views:
        g = _oracle_grads(v)
        seq = g if seq is None else [a + b for a, b in zip(seq, g)]
    for k, a, b in zip(GRAD_KEYS, summed, seq):
        assert a.shape == b.shape, k
        assert float(b.abs().max()) > 0, k
        torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-6 * float(b.abs().max()), msg=k)


@pytest.mark.gpu
def test_sharded_gradient_sum_nccl(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import vi_testlib as tl
    summed = _run("nccl", tmp_path)
    views = _views(torch.device("cuda", 0))
    seq = None
    for v in views:
        g = _cuda_grads(v)
        seq = g if seq is None else [a + b for a, b in zip(seq, g)]
    tl.assert_grads({k: a.numpy() for k, a in zip(GRAD_KEYS, summed)} | {"dL_dmeans3D": np.zeros(3)},
                    {k: b.cpu().numpy() for k, b in zip(GRAD_KEYS, seq)} | {"dL_dmeans3D": np.zeros(3)})


def _coalesce_worker(rank, world, port, out_path):
    import torch.distributed as dist
    from datetime import timedelta
    from volume_integration.distributed import allreduce_gradients
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        g = torch.Generator().manual_seed(rank)
        shapes = [(300, 27), (4096,), (8, 32), (8,)]
        a = [torch.randn(*sh, generator=g) for sh in shapes]
        b = [x.clone() for x in a]
        allreduce_gradients(a, coalesce=False)
        out = allreduce_gradients(b + [None], coalesce=True)
        assert out[-1] is None
        if rank == 0:
            torch.save((a, b), out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_coalesced_allreduce_equals_per_tensor_gloo(tmp_path):
    # one all-reduce over a flat copy of every gradient sums the same values
    # as one all-reduce per tensor, and restores each tensor's shape
    out = str(tmp_path / "coalesced.pt")
    mp.start_processes(_coalesce_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    a, b = torch.load(out)
    for x, y in zip(a, b):
        assert x.shape == y.shape
        torch.testing.assert_close(x, y, rtol=0, atol=0)

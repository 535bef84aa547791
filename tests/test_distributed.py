"""Data-parallel host logic on CPU with two gloo ranks: views are sharded, the texture and position
gradients of each shard are summed across ranks (at the end of the step, from the backward pass's
hooks, or during the next step), and the result equals the gradient of the whole batch on one
process. The CPU oracle stands in for the kernels (the kernels need a GPU)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
import scenes
from diffrast_b200.distributed import (NextStepGradientSum, OverlappedGradientSum, sum_gradients,
                                      view_shard)


def test_view_shard_covers_every_view_once():
    for views in (1, 7, 64):
        for world in (1, 2, 3, 8):
            covered = []
            for rank in range(world):
                covered.extend(range(views)[view_shard(views, rank, world)])
            assert covered == list(range(views))
    with pytest.raises(ValueError):
        view_shard(4, 2, 2)


def _scene():
    pos, tri = scenes.grid_mesh(6, torch.Generator().manual_seed(3), batch=4)
    gen = torch.Generator().manual_seed(4)
    tex = torch.rand(1, 8, 8, 3, generator=gen)
    uv = torch.rand(pos.shape[1], 2, generator=gen)
    target = torch.rand(4, 24, 24, 3, generator=gen)
    return pos, tri, tex, uv, target


def _loss(pos, tri, tex, uv, target):
    rast, rast_db = oracle.rasterize(pos, tri, (24, 24))
    uvp, uv_da = oracle.interpolate(uv, rast, tri, rast_db, [0, 1])
    color = oracle.texture(tex, uvp, uv_da, None, None, "linear-mipmap-linear", "wrap")
    image = oracle.antialias(color, rast, pos, tri)
    # Sum over views (not a mean), so that shard losses add up to the full-batch loss.
    return ((image - target) ** 2).sum()


def _rank(rank: int, world: int, port: int, results) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(1)
        pos, tri, tex, uv, target = _scene()
        shard = view_shard(pos.shape[0], rank, world)
        tex = tex.clone().requires_grad_(True)
        p = pos[shard].clone().requires_grad_(True)
        _loss(p, tri, tex, uv, target[shard]).backward()
        sum_gradients([tex])
        # The same sum with the all-reduce issued from the gradient hook during backward, twice
        # (the reducer is reusable across steps), plus a tensor that gets no gradient.
        tex2 = tex.detach().clone().requires_grad_(True)
        unused = torch.ones(3, requires_grad=True)
        reducer = OverlappedGradientSum([tex2, unused], bucket_bytes=256)
        overlapped = []
        for _ in range(2):
            tex2.grad = None
            _loss(pos[shard].clone(), tri, tex2, uv, target[shard]).backward()
            reducer.wait()
            overlapped.append(tex2.grad.clone())
        reducer.remove()
        # The texture's sum moved to the next step, before its first use: step k's loss is scaled
        # by k + 1, so each sum must be that step's gradient and no other.
        tex3 = tex.detach().clone().requires_grad_(True)
        pipe = NextStepGradientSum(tex3, bucket_bytes=256)
        pipelined = []
        for step in range(3):
            pipe.start()
            pipe.wait()
            if step > 0:
                pipelined.append(pipe.buffer.clone())
            tex3.grad = None
            ((step + 1) * _loss(pos[shard].clone(), tri, tex3, uv, target[shard])).backward()
            pipe.hold()
        pipe.start()
        pipe.wait()
        pipelined.append(pipe.buffer.clone())
        results[rank] = (tex.grad.clone(), shard, p.grad.clone(), overlapped, unused.grad.clone(),
                         pipelined)
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_ranks_sum_to_the_full_batch_gradient():
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_rank, args=(2, _free_port(), results), nprocs=2, start_method="spawn")
    pos, tri, tex, uv, target = _scene()
    tex = tex.clone().requires_grad_(True)
    p = pos.clone().requires_grad_(True)
    _loss(p, tri, tex, uv, target).backward()
    for rank in range(2):
        tex_grad, shard, pos_grad, overlapped, unused_grad, pipelined = results[rank]
        torch.testing.assert_close(tex_grad, tex.grad, atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(pos_grad, p.grad[shard], atol=1e-5, rtol=1e-5)
        for g in overlapped:
            torch.testing.assert_close(g, tex.grad, atol=1e-5, rtol=1e-5)
        assert torch.equal(unused_grad, torch.zeros(3))
        assert len(pipelined) == 3
        for k, g in enumerate(pipelined):
            torch.testing.assert_close(g, (k + 1) * tex.grad, atol=1e-5, rtol=1e-5)

"""Data-parallel host logic on CPU with gloo ranks (world size 2).

* bucketed gradient all-reduce sums every parameter's grad across ranks;
* the GRPO loss with the all-reduced response-token count, summed over ranks, equals
  the single-process loss on the union of the ranks' groups (the reference's global
  token mean, qwen3_grpo_train.py:198), and so do the gradients;
* a rank that fails before the collective makes the others fail with an error within
  the process-group timeout instead of hanging.
"""
import datetime
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ref_ops as R


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _worker_allreduce(rank, world, port, out_dir):
    _init(rank, world, port)
    from qwen3_naive_inference_b200.qwen3_grpo_train import allreduce_grads
    torch.manual_seed(0)
    m = torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.Linear(16, 4))
    for i, p in enumerate(m.parameters()):
        p.grad = torch.full_like(p, float(rank + 1) * (i + 1))
    allreduce_grads(m, bucket_bytes=64)  # several buckets
    torch.save([p.grad for p in m.parameters()], os.path.join(out_dir, f"g{rank}.pt"))
    dist.destroy_process_group()


def _worker_loss(rank, world, port, out_dir):
    _init(rank, world, port)
    data = torch.load(os.path.join(out_dir, "data.pt"))
    rows = data["rows"][rank]
    new = data["new"][rows].clone().requires_grad_(True)
    old, mask, rewards, gids = data["old"][rows], data["mask"][rows], data["rewards"][rows], data["gids"][rows]
    # local advantages (each rank owns whole groups), global denominator via all-reduce
    adv = R.grpo_advantage(rewards, gids)
    total = mask.sum().reshape(1)
    dist.all_reduce(total)
    ratio = (new - old).exp()
    a = adv[:, None] * mask
    lt = -torch.min(ratio * a, ratio.clamp(0.8, 1.2) * a)
    loss = (lt * mask).sum() / (total[0] + 1e-8)
    loss.backward()
    lsum = loss.detach().reshape(1)
    dist.all_reduce(lsum)
    torch.save({"loss": lsum, "grad": new.grad, "rows": rows}, os.path.join(out_dir, f"l{rank}.pt"))
    dist.destroy_process_group()


def _worker_fail(rank, world, port, out_dir):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        os._exit(3)  # dies before joining the collective
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        res = "completed"
    except Exception as e:  # noqa: BLE001 - any error (timeout / connection reset) is the expected outcome
        res = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "fail.txt"), "w") as f:
        f.write(res)
    os._exit(0)


def _spawn(fn, world, out_dir, join=True):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, out_dir)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            raise AssertionError("rank did not finish")
    return [p.exitcode for p in procs]


def test_bucketed_grad_allreduce():
    with tempfile.TemporaryDirectory() as d:
        codes = _spawn(_worker_allreduce, 2, d)
        assert codes == [0, 0]
        g0, g1 = torch.load(os.path.join(d, "g0.pt")), torch.load(os.path.join(d, "g1.pt"))
        for i, (a, b) in enumerate(zip(g0, g1)):
            assert torch.equal(a, b)
            assert torch.all(a == 3.0 * (i + 1))  # (1 + 2) * (i + 1)


def test_global_token_mean_matches_single_process():
    g = torch.Generator().manual_seed(0)
    G, groups, S = 4, 6, 30
    N = G * groups
    rewards = torch.bernoulli(torch.full((N,), 0.5), generator=g)
    gids = torch.arange(groups).repeat_interleave(G)
    new = -torch.rand(N, S, generator=g) * 5
    old = new + 0.05 * torch.randn(N, S, generator=g)
    mask = (torch.rand(N, S, generator=g) > 0.4).float()
    # groups assigned round-robin to ranks, whole groups per rank
    rows = [torch.cat([torch.arange(k * G, (k + 1) * G) for k in range(groups) if k % 2 == r]) for r in range(2)]
    with tempfile.TemporaryDirectory() as d:
        torch.save({"rows": rows, "new": new, "old": old, "mask": mask, "rewards": rewards, "gids": gids},
                   os.path.join(d, "data.pt"))
        assert _spawn(_worker_loss, 2, d) == [0, 0]
        outs = [torch.load(os.path.join(d, f"l{r}.pt")) for r in range(2)]
    loss_ref, grad_ref, _ = R.grpo_loss_and_grad(rewards, gids, new, old, mask)
    assert torch.allclose(outs[0]["loss"], loss_ref.reshape(1), rtol=1e-5)
    grad = torch.zeros_like(new)
    for o in outs:
        grad[o["rows"]] = o["grad"]
    assert torch.allclose(grad, grad_ref, rtol=1e-5, atol=1e-9)


def test_dead_rank_surfaces_as_error_not_hang():
    with tempfile.TemporaryDirectory() as d:
        codes = _spawn(_worker_fail, 2, d)
        assert codes[1] == 3
        with open(os.path.join(d, "fail.txt")) as f:
            assert f.read().startswith("error")

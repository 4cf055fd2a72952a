"""Data parallelism of the fused training pass on the GPU: two ranks (processes sharing cuda:0,
gloo collectives) each run policy_loss_backward on their own prompt groups with the response-token
count and the fp32 gradient buffer summed over ranks; the result equals one process running the
union of the groups (the reference's global token mean, qwen3_grpo_train.py:198): loss and every
gradient.  No kernel waits on another rank, so the two processes can share one GPU."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

TINY = dict(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=128, intermediate_size=256,
            num_hidden_layers=2, vocab_size=512, max_position_embeddings=1024)


def _batch(rows):
    g = torch.Generator().manual_seed(7)
    toks, plens, olds, gids = [], [], [], []
    for gi in range(4):
        prompt = torch.randint(0, 512, (int(torch.randint(20, 60, (1,), generator=g)),), generator=g).tolist()
        for _ in range(2):
            comp = torch.randint(0, 512, (int(torch.randint(5, 40, (1,), generator=g)),), generator=g).tolist()
            toks.append(prompt + comp)
            plens.append(len(prompt))
            olds.append((-6.0 - torch.rand(len(comp), generator=g)).tolist())
            gids.append(gi)
    rewards = torch.tensor([1.0, 0.0, 1.0, 1.0, 0.0, 1.0, 0.0, 0.0])
    sel = list(rows)
    return ([toks[i] for i in sel], [plens[i] for i in sel], [olds[i] for i in sel], rewards[sel],
            [gids[i] for i in sel])


def _run(rows, dev, group=None):
    from qwen3_naive_inference_b200 import ops
    from qwen3_naive_inference_b200 import qwen3_grpo_train as G
    from qwen3_naive_inference_b200.qwen3_naive import Qwen3Config, build_model
    model = build_model(Qwen3Config(**TINY), device=dev, seed=0)
    toks, plens, olds, rewards, gids = _batch(rows)
    batch = G.PackedBatch(toks, plens, olds, rewards, gids, dev, shift=True)
    total = ops.mask_sum(batch.mask)
    if group is not None:
        torch.distributed.all_reduce(total)
    model.zero_grad(set_to_none=True)
    loss, _ = G.policy_loss_backward(model, batch, mask_total=total, microbatch_tokens=96, chunk_rows=40,
                                     process_group=group)
    return loss.cpu(), {n: p.grad.float().cpu() for n, p in model.named_parameters()}


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rows = range(4 * rank, 4 * rank + 4)  # whole groups per rank
    loss, grads = _run(rows, dev, group=torch.distributed.group.WORLD)
    torch.save({"loss": loss, "grads": grads}, os.path.join(out, f"r{rank}.pt"))
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def test_two_ranks_equal_one_process(cuda, tmp_path):
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    single_loss, single = _run(range(8), cuda)
    r0, r1 = torch.load(tmp_path / "r0.pt"), torch.load(tmp_path / "r1.pt")
    # each rank's loss is its groups' share of the global token mean
    assert torch.allclose(r0["loss"] + r1["loss"], single_loss, rtol=1e-4, atol=1e-6)
    for name, g1 in single.items():
        a, b = r0["grads"][name], r1["grads"][name]
        assert torch.equal(a, b), name  # every rank steps on the same all-reduced gradient
        if g1.norm() == 0:
            assert a.norm() == 0, name
            continue
        cos = torch.nn.functional.cosine_similarity(a.reshape(-1), g1.reshape(-1), 0).item()
        assert 1 - cos < 1e-4, (name, cos)
        assert (a - g1).abs().max() <= 2 ** -7 * g1.abs().max() + 1e-6, name  # within bf16 rounding of the sum

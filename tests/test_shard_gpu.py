"""Output-column sharding of one projection (exl3b/shard.py) on the GPU.

One GPU: every rank's column range, quantized alone, is bit-identical to the
same slice of the unsplit quantize_linear (trellis, W_hat rows, svh, Wscale),
at a small shape and at configuration 2 split eight ways.  Two GPUs (run when
present): two NCCL ranks quantize one projection by columns and all-gather it;
the assembled layer equals the one-GPU result bit for bit."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _problem(k, n, seed):
    gen = torch.Generator().manual_seed(seed)
    A = torch.randn(k, k, generator=gen)
    H = A.t() @ A / k + 0.1 * torch.eye(k)
    W = torch.randn(n, k, generator=gen) * 0.02
    return W, H


def _check_slices(W, H, K, worlds):
    from exl3b import api, shard
    n = W.shape[0]
    full = api.quantize_linear(W, H, K=K, out_device="cuda")
    for world in worlds:
        for a, b in shard.column_ranges(n, world):
            part = shard.quantize_linear_columns(W, H, (a, b), K=K, out_device="cuda")
            assert torch.equal(part["trellis"], full["trellis"][:, a // 16:b // 16]), (world, a)
            assert torch.equal(part["W_hat"], full["W_hat"][a:b]), (world, a)
            assert torch.equal(part["svh"], full["svh"][a:b])
            assert part["Wscale"] == full["Wscale"] and part["cols"] == (a, b)


def test_column_ranges_are_slices_of_the_whole_small():
    W, H = _problem(512, 640, 81)
    _check_slices(W, H, 5, (2, 3))


def test_column_ranges_are_slices_of_the_whole_config2():
    from exl3b import synth
    W, H = synth.config2(device="cuda")
    from exl3b import api, shard
    full = api.quantize_linear(W, H, K=4, out_device="cuda")
    for a, b in (shard.column_ranges(5120, 8)[0], shard.column_ranges(5120, 8)[5]):
        part = shard.quantize_linear_columns(W, H, (a, b), K=4, out_device="cuda")
        assert torch.equal(part["trellis"], full["trellis"][:, a // 16:b // 16]), a
        assert torch.equal(part["W_hat"], full["W_hat"][a:b]), a


def _rank_main(rank, world, port, q):
    import numpy as np
    import torch.distributed as dist
    from datetime import timedelta
    from exl3b import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      RANK=str(rank), WORLD_SIZE=str(world))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    W, H = _problem(512, 768, 82)
    out = shard.quantize_linear_split(W, H, K=4, out_device=torch.device("cuda", rank))
    dist.destroy_process_group()
    q.put((rank, out["trellis"].cpu().numpy().copy(), out["W_hat"].cpu().numpy().copy(),
           out["Wscale"]))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_nccl_split_equals_one_gpu():
    from exl3b import api
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    W, H = _problem(512, 768, 82)
    full = api.quantize_linear(W, H, K=4, out_device="cuda")
    for rank, tr, wh, ws in got:
        assert torch.equal(torch.from_numpy(tr), full["trellis"].cpu()), rank
        assert torch.equal(torch.from_numpy(wh), full["W_hat"].cpu()), rank
        assert ws == full["Wscale"]

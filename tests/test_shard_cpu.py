"""Output-column sharding of one projection (exl3b/shard.py) on CPU: the
column ranges are a 128-aligned, complete, balanced partition, and a
world-size-2 gloo run assembles the ranks' ranges (trellis tiles, W_hat rows)
into the whole layer in order, with ranges of unequal width."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from exl3b import shard


@pytest.mark.parametrize("n,world", [(5120, 1), (5120, 2), (5120, 8), (1024, 3), (6144, 5),
                                     (128, 1)])
def test_column_ranges_partition(n, world):
    rs = shard.column_ranges(n, world)
    assert len(rs) == world and rs[0][0] == 0 and rs[-1][1] == n
    for (a, b), (c, _) in zip(rs, rs[1:]):
        assert b == c
    widths = [b - a for a, b in rs]
    assert all(w % 128 == 0 for w in widths)
    assert max(widths) - min(widths) <= 128


def test_column_ranges_rejects_unaligned():
    with pytest.raises(ValueError):
        shard.column_ranges(5000, 2)


def _fake_part(rank, world, n, k, K):
    a, b = shard.column_ranges(n, world)[rank]
    w = b - a
    tr = torch.arange(k // 16 * (w // 16) * 16 * K, dtype=torch.int32).reshape(
        k // 16, w // 16, 16 * K)
    tr = ((tr + 1000 * rank) % 30000).to(torch.int16)
    Wh = torch.full((w, k), float(rank)) + torch.arange(w).unsqueeze(1) / 1000.0
    return {"trellis": tr, "W_hat": Wh, "svh": torch.ones(w).half(), "Wscale": 1.5,
            "K": K, "cols": (a, b)}


def _rank_main(rank, world, port, n, k, K, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    out = shard.gather_columns(_fake_part(rank, world, n, k, K), n)
    dist.destroy_process_group()
    # numpy copies: torch tensors in a queue are shared-memory handles that
    # die with this process
    q.put((rank, out["trellis"].numpy().copy(), out["W_hat"].numpy().copy(), out["cols"],
           tuple(out["svh"].shape)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_gloo_gather_assembles_the_layer():
    world, n, k, K = 2, 384, 256, 3          # ranges 256 + 128 columns (unequal)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n, k, K, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    parts = [_fake_part(r, world, n, k, K) for r in range(world)]
    want_tr = torch.cat([p["trellis"] for p in parts], dim=1)
    want_wh = torch.cat([p["W_hat"] for p in parts], dim=0)
    for rank, tr, wh, cols, svh_shape in got:
        assert torch.equal(torch.from_numpy(tr), want_tr), rank
        assert torch.equal(torch.from_numpy(wh), want_wh), rank
        assert cols == (0, n) and svh_shape == (n,)

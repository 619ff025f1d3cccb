"""Layer-stack sharding across ranks (exl3b/stack.py) on CPU: the layer
assignment is a disjoint, complete, balanced partition, and a world-size-2
gloo run (one process per rank, a host-side stand-in for the per-layer
quantizer) covers every (layer, tensor) exactly once with no data-path
collective, only the final gather of statistics."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from exl3b import stack, synth


@pytest.mark.parametrize("n_layers,world", [(64, 8), (64, 1), (7, 2), (3, 4), (0, 2)])
def test_assign_layers_partition(n_layers, world):
    parts = stack.assign_layers(n_layers, world)
    assert len(parts) == world
    flat = sorted(l for p in parts for l in p)
    assert flat == list(range(n_layers))
    sizes = [len(p) for p in parts]
    assert max(sizes) - min(sizes) <= 1


def _fake_quantize(layer, device, out_root=None):
    return [{"layer": layer, "tensor": name, "weights": o * i, "pid": os.getpid()}
            for name, o, i in synth.STACK_SHAPES]


def _rank_main(rank, world, port, n_layers, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    stats = stack.run_rank(n_layers, rank, world, "cpu", quantize=_fake_quantize)
    gathered = [None] * world
    dist.all_gather_object(gathered, stats)
    dist.destroy_process_group()
    if rank == 0:
        q.put(gathered)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_gloo_stack_covers_every_tensor_once():
    world, n_layers = 2, 5
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n_layers, q))
             for r in range(world)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    seen = [(s["layer"], s["tensor"]) for part in gathered for s in part]
    assert sorted(seen) == sorted((l, n) for l in range(n_layers)
                                  for n, _, _ in synth.STACK_SHAPES)
    # each rank processed only its own layers, in its own process
    for r, part in enumerate(gathered):
        assert {s["layer"] for s in part} == set(stack.assign_layers(n_layers, world)[r])
        assert len({s["pid"] for s in part}) == 1
    assert len({part[0]["pid"] for part in gathered}) == world
    assert sum(s["weights"] for part in gathered for s in part) == \
        n_layers * synth.stack_weights_per_layer()


def test_writer_thread_writes_what_inline_writes(tmp_path):
    """The background writer produces the same files as a direct write."""
    import torch
    from exl3b import export
    gen = torch.Generator().manual_seed(3)
    r = {"trellis": torch.randint(-30000, 30000, (4, 2, 64), generator=gen).to(torch.int16),
         "suh": torch.randn(64, generator=gen).half(), "svh": torch.randn(32, generator=gen).half(),
         "Wscale": 0.75, "K": 4, "code": "exl3_mul1", "channel_scales": False}
    export.save_quantized(tmp_path / "a", 3, "mlp.down_proj", r, meta={"group": "down"})
    w = stack.Writer(tmp_path / "b")
    w.submit(3, "mlp.down_proj", r, {"group": "down"})
    w.close()
    for suffix in (".safetensors", ".json"):
        a = (tmp_path / "a" / "L03" / f"mlp.down_proj{suffix}").read_bytes()
        b = (tmp_path / "b" / "L03" / f"mlp.down_proj{suffix}").read_bytes()
        assert a == b, suffix


def test_writer_reports_a_failed_write(tmp_path):
    import torch
    blocker = tmp_path / "file"
    blocker.write_text("x")                      # a file where the layer dir should go
    w = stack.Writer(blocker)
    r = {"trellis": torch.zeros(1, 1, 32, dtype=torch.int16), "suh": torch.ones(16).half(),
         "svh": torch.ones(16).half(), "Wscale": 1.0, "K": 2}
    w.submit(0, "mlp.up_proj", r, {})
    with pytest.raises(OSError):
        w.close()


def test_hessian_files_in_the_reference_naming(tmp_path):
    import torch
    from safetensors.torch import save_file
    save_file({"H": torch.eye(8)}, str(tmp_path / "L2_mlp.gate_proj.safetensors"))
    save_file({"H": torch.eye(4)}, str(tmp_path / "L3_down.safetensors"))
    p = stack.hessian_path(tmp_path, 2, "mlp", ["gate", "up"])
    assert p.name == "L2_mlp.gate_proj.safetensors"
    assert stack.hessian_path(tmp_path, 3, "down", ["down"]).name == "L3_down.safetensors"
    with pytest.raises(FileNotFoundError):
        stack.hessian_path(tmp_path, 4, "o", ["o"])
    assert torch.equal(stack.load_hessian(p, 8, "cpu"), torch.eye(8))
    with pytest.raises(ValueError):
        stack.load_hessian(p, 16, "cpu")


@pytest.mark.parametrize("world", [1, 2, 3, 4, 7, 8])
def test_layer_ranges_partition(world):
    """Splitting one layer over `world` ranks: every output channel of every
    tensor on exactly one rank, one range per (rank, tensor), ranges
    increasing with the rank, 128-aligned; the chosen cut never predicts a
    slower slowest rank than the plain equal-weight cut, and an equal-weight
    cut keeps each rank within one chunk of the ideal share."""
    plan = stack.layer_ranges(world)
    assert len(plan) == world
    for name, out_f, in_f in synth.STACK_SHAPES:
        got = sorted((a, b, r) for r, rr in enumerate(plan) for m, a, b in rr if m == name)
        assert got[0][0] == 0 and got[-1][1] == out_f
        for (a0, b0, r0), (a1, b1, r1) in zip(got, got[1:]):
            assert b0 == a1 and r1 > r0            # contiguous, one range per rank
        assert all(a % stack.ALIGN == 0 and b % stack.ALIGN == 0 for a, b, _ in got)
    even = stack._cut_plan(world, 0.0)
    assert max(stack._rank_ms(rr) for rr in plan) <= max(stack._rank_ms(rr) for rr in even)
    total = sum(o * i for _n, o, i in synth.STACK_SHAPES)
    biggest = max(stack.ALIGN * i for _n, _o, i in synth.STACK_SHAPES)
    ins = {n: i for n, _o, i in synth.STACK_SHAPES}
    for rr in even:
        mass = sum((b - a) * ins[m] for m, a, b in rr)
        assert abs(mass - total / world) <= biggest, (mass, total / world)


def test_layer_ranges_avoid_narrow_long_chains():
    """At 4 and 8 ranks no rank holds a narrow remnant of the down projection
    (1088 sequential k-blocks) on top of other work."""
    for world in (4, 8):
        for rr in stack.layer_ranges(world):
            downs = [(a, b) for m, a, b in rr if m == "down"]
            if downs and len(rr) > 1:
                assert all(b - a >= 1024 for a, b in downs), rr


# a small stand-in layer for the gloo run of the split layer's gather
_SMALL_SHAPES = [("q", 384, 256), ("k", 128, 256), ("v", 128, 256), ("o", 256, 384),
                 ("gate", 512, 256), ("up", 512, 256), ("down", 256, 512)]
_SMALL_GROUPS = [("attn", 256, ["q", "k", "v"]), ("o", 384, ["o"]),
                 ("mlp", 256, ["gate", "up"]), ("down", 512, ["down"])]


def _tile_code(name, in_f, n0, n1, K):
    """Deterministic stand-in trellis of channels [n0, n1) of `name`."""
    import torch
    idx = [n for n, _o, _i in _SMALL_SHAPES].index(name)
    tk, cols = in_f // 16, torch.arange(n0 // 16, n1 // 16)
    t = (torch.arange(tk)[:, None, None] * 7 + cols[None, :, None] * 131
         + torch.arange(16 * K)[None, None, :] + 1000 * idx)
    return (t % 30000).to(torch.int16)


def _split_rank_main(rank, world, port, out, q):
    import torch
    import torch.distributed as dist
    from exl3b import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    synth.STACK_SHAPES[:] = _SMALL_SHAPES
    synth.STACK_GROUPS[:] = _SMALL_GROUPS
    seen = []

    def fake_fused(pieces, Lfac, out_device=None, **kw):
        out = []
        for (name, in_f), cols, K in pieces:
            seen.append((name, cols))
            out.append({"trellis": _tile_code(name, in_f, cols[0], cols[1], K),
                        "Wscale": 0.5 + [n for n, _o, _i in _SMALL_SHAPES].index(name)})
        return out

    shard.quantize_columns_fused = fake_fused
    shard.lfac = lambda H, k, **kw: None
    synth.hessian = lambda dim, seed, device: None
    synth.stack_weight = lambda layer, m, device: (m, {n: i for n, _o, i in _SMALL_SHAPES}[m])
    stats = stack.quantize_layer_split(3, "cpu", out_root=out if rank == 0 else None)
    dist.destroy_process_group()
    q.put((rank, seen, stats))


def test_two_rank_gloo_layer_split_assembles_every_tensor(tmp_path):
    """A layer split over two gloo ranks (a small stand-in layer, the per-range
    quantizer replaced by a deterministic code): each rank quantizes only its
    planned ranges, and rank 0 writes every tensor whole, its trellis the
    ranks' pieces side by side and its scale the tensor's."""
    from exl3b import export
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_split_rank_main, args=(r, world, port, str(tmp_path), q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = dict((r, (seen, st)) for r, seen, st in (q.get(timeout=180) for _ in range(world)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    orig_shapes = list(synth.STACK_SHAPES)
    synth.STACK_SHAPES[:] = _SMALL_SHAPES
    try:
        plan = stack.layer_ranges(world)
    finally:
        synth.STACK_SHAPES[:] = orig_shapes
    for r in range(world):
        assert sorted(got[r][0]) == sorted((m, (a, b)) for m, a, b in plan[r])
    assert got[1][1] == [] and len(got[0][1]) == len(_SMALL_SHAPES)
    for idx, (name, out_f, in_f) in enumerate(_SMALL_SHAPES):
        f = export.load_quantized(tmp_path / "L03" / f"{stack.MODULE_NAMES[name]}.safetensors")
        K = synth.SC5_K[name]
        assert f["trellis"].shape == (in_f // 16, out_f // 16, 16 * K)
        assert (f["trellis"] == _tile_code(name, in_f, 0, out_f, K)).all()
        assert f["meta"]["Wscale"] == 0.5 + idx and f["meta"]["split_ranks"] == world

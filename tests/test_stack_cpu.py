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

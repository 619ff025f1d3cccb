"""Layer-stack driver: quantize a stack of transformer layers (the 27B-shape
mixed-K stack of config 5) on the GPUs of one node, one process per GPU.

Sharding: whole layers per rank (layer l -> rank l mod world).  Every layer
has the same shapes and the ACS count per weight does not depend on K, so
whole layers balance evenly; a layer's k-sweep is sequential and never split.
Ranks exchange nothing while quantizing: each reads its own synthetic
weights / Hessians (seeded by layer and tensor) and writes its tensors'
EXL3 files (exl3b.export layout) into the shared output directory.  The
only collective is the gather of per-rank statistics at the end, outside the
quantization.

Within a layer, tensors that read the same activations share one Hessian and
form one fused module (q/k/v, gate/up), quantized by quantize_linear_fused
at their per-member K (synth.SC5_K by default).

    torchrun --nproc-per-node 8 -m exl3b.stack --layers 64 --out DIR
"""
from __future__ import annotations

import argparse
import json
import os
import time

MODULE_NAMES = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj",
                "o": "self_attn.o_proj", "gate": "mlp.gate_proj", "up": "mlp.up_proj",
                "down": "mlp.down_proj"}


def assign_layers(n_layers: int, world: int) -> list:
    """Layers of each rank: layer l -> rank l mod world."""
    if world < 1 or n_layers < 0:
        raise ValueError("world >= 1, n_layers >= 0")
    return [list(range(r, n_layers, world)) for r in range(world)]


def quantize_layer(layer: int, device, Ks: dict | None = None, out_root=None,
                   tensors: list | None = None) -> list:
    """Quantize one layer's tensors on `device`; returns per-tensor stats
    (name, K, weights, Wscale, seconds).  Writes EXL3 files when out_root is
    given."""
    import torch

    from . import api, export, synth
    Ks = dict(synth.SC5_K if Ks is None else Ks)
    stats = []
    for group, dim, members in synth.STACK_GROUPS:
        members = [m for m in members if tensors is None or m in tensors]
        if not members:
            continue
        t0 = time.time()
        H = synth.hessian(dim, synth.stack_hessian_seed(layer, group), device)
        Ws = [synth.stack_weight(layer, m, device) for m in members]
        res = api.quantize_linear_fused(Ws, H, Ks=[Ks[m] for m in members], device=device,
                                        out_device=device)
        torch.cuda.synchronize(device)
        dt = time.time() - t0
        for m, W, r in zip(members, Ws, res):
            if out_root is not None:
                export.save_quantized(out_root, layer, MODULE_NAMES[m], r,
                                      meta={"group": group, "layer": layer})
            stats.append({"layer": layer, "tensor": m, "K": r["K"],
                          "weights": W.numel(), "Wscale": r["Wscale"],
                          "seconds": dt * W.numel() / sum(w.numel() for w in Ws)})
        del H, Ws, res
    return stats


def run_rank(n_layers: int, rank: int, world: int, device, out_root=None,
             quantize=quantize_layer, **kw) -> list:
    """This rank's share of the stack; `quantize(layer, device, ...)` returns
    per-tensor stats."""
    stats = []
    for layer in assign_layers(n_layers, world)[rank]:
        stats.extend(quantize(layer, device, out_root=out_root, **kw))
    return stats


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=64)
    ap.add_argument("--out", default=None, help="EXL3 per-tensor output root (optional)")
    ap.add_argument("--tensors", default=None, help="comma list of tensors (default all)")
    a = ap.parse_args(argv)
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    tensors = a.tensors.split(",") if a.tensors else None
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier(device_ids=[local])
    torch.cuda.synchronize()
    ev0.record()
    stats = run_rank(a.layers, rank, world, dev, a.out, tensors=tensors)
    ev1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([ev0.elapsed_time(ev1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        gathered = [None] * world
        dist.all_gather_object(gathered, stats)
        stats = [s for part in gathered for s in part]
        dist.destroy_process_group()
    if rank == 0:
        weights = sum(s["weights"] for s in stats)
        print(json.dumps({"layers": a.layers, "n_gpus": world, "tensors": len(stats),
                          "weights": weights, "seconds": float(ms.item()) / 1e3,
                          "weights_per_s": weights / (float(ms.item()) / 1e3)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

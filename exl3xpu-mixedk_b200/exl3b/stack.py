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

Inputs: seeded synthetic weights; Hessians either synthetic (seeded per layer
and group) or read from a directory of captured input Grams in the
reference's dump format (check_tensor_bitexact.py:25-30, 94-95): one
safetensors file per layer and linear, key "H", the undamped [in, in] Gram,
named L{layer}_{module}.safetensors after the group's first member (e.g.
L2_mlp.gate_proj.safetensors for gate/up) or L{layer}_{group}.safetensors.

Timing: the synthesis (or loading) of each group's inputs and its
quantization are timed separately with CUDA events.  Finished tensors leave
the device as their three stored EXL3 fields and are written to disk by a
background thread, so the file I/O overlaps the next group's quantization.

    torchrun --nproc-per-node 8 -m exl3b.stack --layers 64 --out DIR [--hessians HDIR]
"""
from __future__ import annotations

import argparse
import json
import os
import queue
import threading
import time
from pathlib import Path

MODULE_NAMES = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj",
                "o": "self_attn.o_proj", "gate": "mlp.gate_proj", "up": "mlp.up_proj",
                "down": "mlp.down_proj"}


def assign_layers(n_layers: int, world: int) -> list:
    """Layers of each rank: layer l -> rank l mod world."""
    if world < 1 or n_layers < 0:
        raise ValueError("world >= 1, n_layers >= 0")
    return [list(range(r, n_layers, world)) for r in range(world)]


class Writer:
    """Background writer of per-tensor EXL3 files: submit() queues the stored
    fields (CPU tensors) of one tensor, a thread writes them with
    export.save_quantized; close() waits for the queue to drain and re-raises
    the first write error."""

    def __init__(self, root):
        self.root = root
        self.q: queue.Queue = queue.Queue(maxsize=16)
        self.err = None
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        from . import export
        while True:
            item = self.q.get()
            if item is None:
                return
            if self.err is None:
                try:
                    export.save_fields(self.root, *item)
                except Exception as e:          # reported by close()
                    self.err = e

    def submit(self, layer: int, module: str, result: dict, meta: dict):
        from . import export
        # device -> host in the calling thread (its stream order); the file
        # I/O in the writer thread
        self.q.put((layer, module, export.stored_fields(result),
                    export.tensor_info(module, result, meta)))

    def close(self):
        self.q.put(None)
        self.t.join()
        if self.err is not None:
            raise self.err


def hessian_path(hdir, layer: int, group: str, members: list) -> Path:
    """The captured Gram of (layer, group) under hdir, in the reference's
    naming: L{layer}_{module}.safetensors of the group's first member, or
    L{layer}_{group}.safetensors."""
    cands = [Path(hdir) / f"L{layer}_{MODULE_NAMES[members[0]]}.safetensors",
             Path(hdir) / f"L{layer}_{group}.safetensors"]
    for c in cands:
        if c.exists():
            return c
    raise FileNotFoundError(f"no Hessian for layer {layer} group {group!r}: tried "
                            f"{', '.join(str(c) for c in cands)}")


def load_hessian(path, dim: int, device):
    """Key "H" of a Gram dump: fp32 [dim, dim] on `device`."""
    from safetensors.torch import load_file
    H = load_file(str(path))["H"]
    if tuple(H.shape) != (dim, dim):
        raise ValueError(f"{path}: H is {tuple(H.shape)}, the group's input dim is {dim}")
    import torch
    return H.to(device=device, dtype=torch.float32)


def quantize_layer(layer: int, device, Ks: dict | None = None, out_root=None,
                   tensors: list | None = None, writer: Writer | None = None,
                   hessian_dir=None) -> list:
    """Quantize one layer's tensors on `device`; returns per-tensor stats
    (name, K, weights, Wscale, seconds of quantization, seconds of input
    synthesis / loading -- each group's time shared by weight).  Writes EXL3
    files when out_root is given (through `writer` in the background, else
    inline)."""
    import torch

    from . import api, export, synth
    Ks = dict(synth.SC5_K if Ks is None else Ks)
    stats = []
    s = torch.cuda.current_stream(device)
    for group, dim, group_members in synth.STACK_GROUPS:
        members = [m for m in group_members if tensors is None or m in tensors]
        if not members:
            continue
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(s)
        if hessian_dir is not None:
            H = load_hessian(hessian_path(hessian_dir, layer, group, group_members), dim,
                             device)
        else:
            H = synth.hessian(dim, synth.stack_hessian_seed(layer, group), device)
        Ws = [synth.stack_weight(layer, m, device) for m in members]
        ev[1].record(s)
        res = api.quantize_linear_fused(Ws, H, Ks=[Ks[m] for m in members], device=device,
                                        out_device=device)
        ev[2].record(s)
        ev[2].synchronize()
        t_syn, t_q = ev[0].elapsed_time(ev[1]) / 1e3, ev[1].elapsed_time(ev[2]) / 1e3
        tot = sum(w.numel() for w in Ws)
        for m, W, r in zip(members, Ws, res):
            meta = {"group": group, "layer": layer}
            if writer is not None:
                writer.submit(layer, MODULE_NAMES[m], r, meta)
            elif out_root is not None:
                export.save_quantized(out_root, layer, MODULE_NAMES[m], r, meta=meta)
            stats.append({"layer": layer, "tensor": m, "K": r["K"],
                          "weights": W.numel(), "Wscale": r["Wscale"],
                          "seconds": t_q * W.numel() / tot,
                          "synth_seconds": t_syn * W.numel() / tot})
        del H, Ws, res
    return stats


ALIGN = 128


# Time model of one rank's share of a split layer (ms), used only to choose
# between candidate cuts.  A group's sweep over `cols` column tiles and tk
# k-blocks takes about max(tk x CHAIN_MS, tk x cols / TILES_PER_MS): a column's
# k-blocks are sequential, and a k-block of a narrow sweep (tiles alone on
# their SMs, the one-tile-per-CTA kernel) takes ~0.6 ms (B200, in = 5120, 32
# column tiles: K = 4 0.593, K = 5 0.603, K = 6 0.658, K = 7 0.642 ms per
# k-block; K = 4 at 128 column tiles 0.641), while a full-width sweep retires
# ~278 tiles per ms on 148 SMs (config 2: 102400 tiles in 368 ms).  Plus the
# group's Hessian synthesis and block LDL (~31 ms at in = 17408, ~7 ms below).
CHAIN_MS = 0.6
TILES_PER_MS = 278.0


def _rank_ms(ranges) -> float:
    from . import synth
    ins = {n: i for n, _o, i in synth.STACK_SHAPES}
    group = {m: g for g, _d, ms in synth.STACK_GROUPS for m in ms}
    cols = {}
    for m, a, b in ranges:
        g = group[m]
        cols[g] = (cols.get(g, (0, ins[m]))[0] + (b - a) // 16, ins[m])
    return sum(max(k // 16 * CHAIN_MS, k // 16 * c / TILES_PER_MS) + (31 if k >= 16384 else 7)
               for c, k in cols.values())


def _cut_plan(world: int, snap: float) -> list:
    from . import synth
    chunks = [(name, n0, ALIGN * in_f) for name, out_f, in_f in synth.STACK_SHAPES
              for n0 in range(0, out_f, ALIGN)]
    total = sum(c[2] for c in chunks)
    share = total / world
    bounds, acc = [0], 0
    for _name, out_f, in_f in synth.STACK_SHAPES:
        acc += out_f * in_f
        bounds.append(acc)
    cuts = []
    for r in range(1, world):
        c = r * share
        for lo, hi in zip(bounds, bounds[1:]):
            if lo < c < hi:
                if c - lo < snap * share:
                    c = lo
                elif hi - c < snap * share:
                    c = hi
        cuts.append(c)
    parts = [[] for _ in range(world)]
    acc = 0
    for name, n0, mass in chunks:
        r = sum(1 for c in cuts if acc + mass / 2 > c)
        acc += mass
        parts[r].append((name, n0))
    out = []
    for part in parts:
        ranges = []
        for name, n0 in part:
            if ranges and ranges[-1][0] == name and ranges[-1][2] == n0:
                ranges[-1] = (name, ranges[-1][1], n0 + ALIGN)
            else:
                ranges.append((name, n0, n0 + ALIGN))
        out.append(ranges)
    return out


def layer_ranges(world: int) -> list:
    """Per rank, the (tensor, n0, n1) output-channel ranges of one layer of
    the stack when the layer itself is split over `world` ranks.  The layer's
    tensors in order (synth.STACK_SHAPES) form one sequence of 128-channel
    chunks, a chunk of tensor m weighing 128 x in_m weights (the work per
    weight does not depend on K), cut into `world` contiguous parts: at equal
    weight, or with each cut moved to the nearest tensor boundary when it
    would leave a piece smaller than a fraction of the share (a narrow piece
    costs its whole chain of k-blocks: the down projection's 1088 take ~1 s
    at any width).  Of the candidate cuts the one with the least predicted
    time of the slowest rank is taken (_rank_ms).  Every channel belongs to
    exactly one rank, a rank's channels of one tensor form one range, and
    ranks hold increasing ranges (a rank may hold none)."""
    if world < 1:
        raise ValueError("world >= 1")
    best = None
    for snap in (0.0, 0.15, 0.3, 0.5):
        plan = _cut_plan(world, snap)
        cost = max(_rank_ms(rr) for rr in plan)
        if best is None or cost < best[0]:
            best = (cost, plan)
    return best[1]


def quantize_layer_split(layer: int, device, group=None, Ks: dict | None = None,
                         writer: Writer | None = None, out_root=None,
                         hessian_dir=None) -> list:
    """One layer of the stack with its output channels spread over the ranks
    of `group` (layer_ranges; a single process is a world of one).  Each rank
    factors the Hessian of every input group it touches once, quantizes its
    channel ranges of each group in one sweep (shard.quantize_columns_fused:
    bit-identical to the same channels of the unsplit tensors, self-checked),
    and the finished trellises and scales are all-gathered (NCCL).  Rank 0
    assembles each tensor and writes its EXL3 files; returns its per-tensor
    stats there, [] on the other ranks."""
    import torch
    import torch.distributed as dist

    from . import api, export, shard, synth
    Ks = dict(synth.SC5_K if Ks is None else Ks)
    split = dist.is_available() and dist.is_initialized()
    rank = dist.get_rank(group) if split else 0
    world = dist.get_world_size(group) if split else 1
    plan = layer_ranges(world)
    mine = plan[rank]
    parts = {}
    for gname, dim, members in synth.STACK_GROUPS:
        todo = [(m, a, b) for m, a, b in mine if m in members]
        if not todo:
            continue
        if hessian_dir is not None:
            H = load_hessian(hessian_path(hessian_dir, layer, gname, members), dim, device)
        else:
            H = synth.hessian(dim, synth.stack_hessian_seed(layer, gname), device)
        L = shard.lfac(H, dim, device=device)
        del H
        pieces = [(synth.stack_weight(layer, m, device), (a, b), Ks[m]) for m, a, b in todo]
        for (m, _a, _b), r in zip(todo, shard.quantize_columns_fused(pieces, L,
                                                                     out_device=device)):
            parts[m] = r
        del L, pieces
    stats = []
    for name, out_f, in_f in synth.STACK_SHAPES:
        K = Ks[name]
        widths = [sum(b - a for m, a, b in rr if m == name) for rr in plan]
        p = parts.get(name)
        if world > 1:
            wmax = max(widths)
            buf = torch.zeros(in_f // 16, wmax // 16, 16 * K, dtype=torch.int16, device=device)
            if p is not None:
                buf[:, :p["trellis"].shape[1]] = p["trellis"]
            # collectives have no int16 type: the trellis travels as its bytes
            got = [torch.empty_like(buf.view(torch.uint8)) for _ in range(world)]
            dist.all_gather(got, buf.view(torch.uint8), group=group)
            sc = torch.tensor([p["Wscale"] if p is not None else 0.0], dtype=torch.float64,
                              device=device)
            scs = [torch.empty_like(sc) for _ in range(world)]
            dist.all_gather(scs, sc, group=group)
            if rank != 0:
                continue
            trellis = torch.cat([g.view(torch.int16)[:, :w // 16]
                                 for g, w in zip(got, widths) if w], dim=1)
            wscale = float(next(float(x.item()) for x, w in zip(scs, widths) if w))
        else:
            trellis, wscale = p["trellis"], p["Wscale"]
        res = {"trellis": trellis, "suh": api.sign_vec(in_f, 20261011).half(),
               "svh": api.sign_vec(out_f, 20261012).half(), "Wscale": wscale, "K": K,
               "code": "exl3_mul1", "channel_scales": False}
        meta = {"group": next(g for g, _d, ms in synth.STACK_GROUPS if name in ms),
                "layer": layer, "split_ranks": world}
        if writer is not None:
            writer.submit(layer, MODULE_NAMES[name], res, meta)
        elif out_root is not None:
            export.save_quantized(out_root, layer, MODULE_NAMES[name], res, meta=meta)
        stats.append({"layer": layer, "tensor": name, "K": K, "weights": out_f * in_f,
                      "Wscale": wscale})
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
    ap.add_argument("--split-layers", action="store_true",
                    help="split every layer over all ranks (per-layer latency) instead of "
                         "whole layers per rank")
    ap.add_argument("--hessians", default=None,
                    help="directory of captured input Grams (L{layer}_{module}.safetensors, "
                         "key H); default: seeded synthetic Hessians")
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
    writer = Writer(a.out) if a.out else None
    ev0.record()
    if a.split_layers:
        if tensors is not None:
            raise SystemExit("--split-layers quantizes whole layers (no --tensors)")
        stats = []
        for layer in range(a.layers):
            stats.extend(quantize_layer_split(layer, dev, writer=writer if rank == 0 else None,
                                              hessian_dir=a.hessians))
        for st in stats:
            st.setdefault("seconds", 0.0)
            st.setdefault("synth_seconds", 0.0)
    else:
        stats = run_rank(a.layers, rank, world, dev, a.out, tensors=tensors, writer=writer,
                         hessian_dir=a.hessians)
    if writer is not None:
        writer.close()          # the rank's last files are on disk inside the timing
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
        q_s = sum(s["seconds"] for s in stats)
        syn_s = sum(s["synth_seconds"] for s in stats)
        print(json.dumps({"layers": a.layers, "n_gpus": world, "tensors": len(stats),
                          "weights": weights, "seconds": float(ms.item()) / 1e3,
                          "weights_per_s": weights / (float(ms.item()) / 1e3),
                          "quantize_gpu_seconds_all_ranks": q_s,
                          "input_synthesis_gpu_seconds_all_ranks": syn_s,
                          "seconds_per_layer": float(ms.item()) / 1e3 / max(a.layers, 1),
                          "sharding": "each layer split over all ranks" if a.split_layers
                                      else "whole layers per rank",
                          "hessians": a.hessians or "synthetic"}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

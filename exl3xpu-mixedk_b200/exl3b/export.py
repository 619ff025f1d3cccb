"""EXL3 on-disk layout: per-tensor files, fused mixed-K member layout, and
assembly of a complete EXL3 model directory from a template.

Per-tensor input layout (quantize/export_exl3.py:4-8 of the reference):

    ROOT/L{nn}/{module}.safetensors   trellis int16 [k/16, n/16, 16*K]
                                      suh fp16 [k], svh fp16 [n]
    ROOT/L{nn}/{module}.json          {"module": ..., "K": ..., "Wscale": ...}

``module`` is the key suffix inside the model, e.g. "mlp.down_proj" ->
``model.language_model.layers.{nn}.mlp.down_proj.{trellis,suh,svh}``.

Stored scale convention (quantize.py:855-858, 994-1003): the per-tensor
Wscale rides in suh, so ``weight_orig(trellis, suh, svh)`` -- decode, then
diag(suh) B_k . W_inner . B_n diag(svh) -- is the dequantised weight.  The
channel-scales path of quantize_linear already returns folded fp16 suh/svh;
for the plain path the writer folds ``suh * Wscale`` (fp16).

Assembly (export_exl3.py:83-149): every template safetensors shard is copied
and each blob for a provided key is overwritten in place (the header is kept,
so writing a template's own tensors back reproduces it byte for byte); every
other file is copied verbatim; ARTIFACTS.sha256 is regenerated.

Fused mixed-K modules (serve/patches/0002-vllm-plugin-mixed-k.patch:126-205):
members of one fused module (q/k/v, gate/up) are written as separate tensors
with their own K; a consumer that loads them into one module lays the members
out as one flat int16 buffer, member j's [k/16, n_j/16, 16*K_j] block at
offset tseg[j] (``fused_segments`` / ``pack_fused``)."""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import struct
from pathlib import Path

import numpy as np
import torch

QUANT_FIELDS = ("trellis", "suh", "svh")
LAYER_PREFIX = "model.language_model.layers."
# safetensors dtype tags <-> numpy dtypes (the ones the EXL3 fields use, plus
# the common others a template may hold)
_ST_OF_NP = {"int16": "I16", "float16": "F16", "float32": "F32", "int32": "I32",
             "int64": "I64", "uint8": "U8", "bool": "BOOL", "int8": "I8",
             "float64": "F64"}


# ------------------------------------------------------------------ headers
def read_st_header(path) -> tuple[dict, int]:
    """(header dict, byte offset of the data section) of a safetensors file:
    u64 little-endian header length, then that many bytes of JSON."""
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        return json.loads(f.read(hlen)), 8 + hlen


def tensor_bytes(path, key: str) -> bytes:
    """Raw data bytes of one tensor inside a safetensors file."""
    hdr, base = read_st_header(path)
    lo, hi = hdr[key]["data_offsets"]
    with open(path, "rb") as f:
        f.seek(base + lo)
        return f.read(hi - lo)


# ------------------------------------------------------------------ per tensor
def stored_fields(result: dict) -> dict:
    """The three EXL3 fields of one quantize_linear result, on the CPU, with
    the per-tensor scale folded into suh."""
    trellis = result["trellis"].detach().cpu().to(torch.int16).contiguous()
    suh = result["suh"].detach().cpu()
    svh = result["svh"].detach().cpu()
    if not result.get("channel_scales", False):
        suh = suh.float() * float(result["Wscale"])
    return {"trellis": trellis, "suh": suh.half().contiguous(),
            "svh": svh.half().contiguous()}


def save_quantized(root, layer: int, module: str, result: dict,
                   meta: dict | None = None) -> Path:
    """Write ROOT/L{layer:02d}/{module}.safetensors (+ .json metadata) for one
    quantized tensor.  Returns the safetensors path."""
    from safetensors.torch import save_file
    ldir = Path(root) / f"L{int(layer):02d}"
    ldir.mkdir(parents=True, exist_ok=True)
    path = ldir / f"{module}.safetensors"
    save_file(stored_fields(result), str(path))
    info = {"module": module, "K": int(result["K"]), "Wscale": float(result["Wscale"]),
            "code": result.get("code", "exl3_mul1"),
            "channel_scales": bool(result.get("channel_scales", False))}
    if meta:
        info.update(meta)
    path.with_suffix(".json").write_text(json.dumps(info, sort_keys=True))
    return path


def load_quantized(path) -> dict:
    """Read one per-tensor file back: {"trellis", "suh", "svh"} tensors plus
    the metadata json (if present) under "meta"."""
    from safetensors.torch import load_file
    path = Path(path)
    out = dict(load_file(str(path)))
    jp = path.with_suffix(".json")
    out["meta"] = json.loads(jp.read_text()) if jp.exists() else {}
    return out


def weight_orig(trellis: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, K: int,
                code: str = "exl3_mul1", device="cuda") -> torch.Tensor:
    """Dequantise stored EXL3 fields on the device: W_orig [k, n] =
    diag(suh) B_k decode(trellis) B_n diag(svh) (the EXL3 reconstruction the
    reference checks its W_hat against, export_exl3.py:175-199).  Transposed
    relative to the nn.Linear weight [out, in]."""
    from . import api
    k = trellis.shape[0] * 16
    n = trellis.shape[1] * 16
    dev = torch.device(device)
    dec = api.decode_trellis(trellis.to(dev), api.get_lut(code, device=dev), K, k, n)
    return api.from_inner(dec, suh.to(dev), svh.to(dev))


# ------------------------------------------------------------------ fused members
def fused_segments(k: int, n_sizes: list, Ks: list) -> list:
    """Start offsets (int16 elements) of each member's [k/16, n_j/16, 16*K_j]
    block in the flat packed trellis of a mixed-K fused module, plus the total
    length as the last entry (one member per output partition)."""
    if len(n_sizes) != len(Ks):
        raise ValueError("one K per member")
    offs = [0]
    for n_j, K_j in zip(n_sizes, Ks):
        if k % 16 or n_j % 16:
            raise ValueError("k and n_j must be multiples of 16")
        offs.append(offs[-1] + (k // 16) * (n_j // 16) * 16 * int(K_j))
    return offs


def pack_fused(trellises: list) -> torch.Tensor:
    """Flat int16 buffer holding each member's trellis at its segment."""
    return torch.cat([t.reshape(-1).to(torch.int16) for t in trellises])


def unpack_fused(flat: torch.Tensor, k: int, n_sizes: list, Ks: list) -> list:
    offs = fused_segments(k, n_sizes, Ks)
    if flat.numel() != offs[-1]:
        raise ValueError(f"flat trellis has {flat.numel()} elements, layout needs {offs[-1]}")
    return [flat[offs[j]:offs[j + 1]].reshape(k // 16, n // 16, 16 * K)
            for j, (n, K) in enumerate(zip(n_sizes, Ks))]


# ------------------------------------------------------------------ assembly
def collect_inputs(tensors_root) -> dict:
    """key -> (dtype tag, shape, raw bytes) for every per-tensor file under
    ROOT/L*/ (key = model.language_model.layers.{nn}.{module}.{field})."""
    from safetensors import safe_open
    out = {}
    for st_path in sorted(Path(tensors_root).glob("L*/*.safetensors")):
        nn = str(int(st_path.parent.name[1:]))
        module = st_path.stem
        jp = st_path.with_suffix(".json")
        if jp.exists():
            module = json.loads(jp.read_text()).get("module", module)
        prefix = f"{LAYER_PREFIX}{nn}.{module}."
        with safe_open(str(st_path), framework="np") as f:
            present = set(f.keys())
            for field in QUANT_FIELDS:
                if field not in present:
                    raise KeyError(f"{st_path}: missing key {field!r} (has {sorted(present)})")
                arr = f.get_tensor(field)
                tag = _ST_OF_NP.get(str(arr.dtype))
                if tag is None:
                    raise ValueError(f"{st_path}:{field} has unsupported dtype {arr.dtype}")
                out[prefix + field] = (tag, list(arr.shape), np.ascontiguousarray(arr).tobytes())
    return out


def _sha256_tree(outdir: Path) -> None:
    lines = []
    for item in sorted(outdir.iterdir()):
        if not item.is_file() or item.name == "ARTIFACTS.sha256":
            continue
        h = hashlib.sha256()
        with open(item, "rb") as f:
            while True:
                buf = f.read(1 << 24)
                if not buf:
                    break
                h.update(buf)
        lines.append(f"{h.hexdigest()}  {item.name}")
    (outdir / "ARTIFACTS.sha256").write_text("\n".join(lines) + "\n")


def export(tensors_root, template, outdir) -> int:
    """Assemble a complete EXL3 model directory: the template with every
    provided tensor's blob replaced in place.  Returns the number of blobs
    replaced.  Raises on a key the template does not have, a dtype / shape /
    size mismatch, or a key left unwritten."""
    template, outdir = Path(template), Path(outdir)
    weight_map = json.loads((template / "model.safetensors.index.json").read_text())["weight_map"]
    inputs = collect_inputs(tensors_root)
    by_shard: dict = {}
    for key, val in inputs.items():
        if key not in weight_map:
            raise KeyError(f"input key {key} not in template index")
        by_shard.setdefault(weight_map[key], {})[key] = val
    outdir.mkdir(parents=True, exist_ok=True)
    shards = sorted(set(weight_map.values()))
    written = set()
    for shard in shards:
        src, dst = template / shard, outdir / shard
        hdr, base = read_st_header(src)
        repl = by_shard.get(shard, {})
        for key, (tag, shape, raw) in repl.items():
            ent = hdr[key]
            if ent["dtype"] != tag:
                raise ValueError(f"{key}: dtype {tag} != template {ent['dtype']}")
            if list(ent["shape"]) != shape:
                raise ValueError(f"{key}: shape {shape} != template {ent['shape']}")
            lo, hi = ent["data_offsets"]
            if hi - lo != len(raw):
                raise ValueError(f"{key}: {len(raw)} bytes != template {hi - lo}")
        shutil.copyfile(src, dst)
        if repl:
            with open(dst, "r+b") as f:
                for key, (_tag, _shape, raw) in repl.items():
                    f.seek(base + hdr[key]["data_offsets"][0])
                    f.write(raw)
                    written.add(key)
    left = set(inputs) - written
    if left:
        raise RuntimeError(f"keys not written: {sorted(left)}")
    shard_set = set(shards)
    for item in template.iterdir():
        if item.is_file() and item.name not in shard_set and item.name != "ARTIFACTS.sha256":
            shutil.copyfile(item, outdir / item.name)
    _sha256_tree(outdir)
    return len(written)


def extract_template(template, workdir, only_keys=None) -> tuple[Path, int]:
    """Write a template's own decoder-layer EXL3 tensors into the per-tensor
    input layout under WORKDIR/tensors (the inverse of export; used for the
    byte-identical round trip).  Returns (root, number of files)."""
    from safetensors.torch import save_file
    template = Path(template)
    weight_map = json.loads((template / "model.safetensors.index.json").read_text())["weight_map"]
    root = Path(workdir) / "tensors"
    files: dict = {}
    np2t = {"I16": torch.int16, "F16": torch.float16, "F32": torch.float32,
            "I32": torch.int32, "BF16": torch.bfloat16, "I64": torch.int64,
            "U8": torch.uint8, "BOOL": torch.bool}
    for key, shard in weight_map.items():
        if not key.startswith(LAYER_PREFIX) or not key.endswith(QUANT_FIELDS):
            continue
        if only_keys is not None and key not in only_keys:
            continue
        parts = key[len(LAYER_PREFIX):].split(".")
        nn, field, module = parts[0], parts[-1], ".".join(parts[1:-1])
        st = root / f"L{nn}" / f"{module}.safetensors"
        hdr, _ = read_st_header(template / shard)
        ent = hdr[key]
        raw = bytearray(tensor_bytes(template / shard, key))
        t = torch.frombuffer(raw, dtype=np2t[ent["dtype"]]).reshape(ent["shape"]).clone()
        files.setdefault(st, {})[field] = t
    for st, fields in files.items():
        st.parent.mkdir(parents=True, exist_ok=True)
        save_file(fields, str(st))
        K = int(fields["trellis"].shape[-1] // 16) if "trellis" in fields else 0
        st.with_suffix(".json").write_text(json.dumps({"module": st.stem, "K": K}))
    return root, len(files)


def check_keys(template, outdir) -> list:
    """Template keys missing from the output, or present with another
    dtype / shape: list of (key, problem)."""
    template, outdir = Path(template), Path(outdir)
    tmap = json.loads((template / "model.safetensors.index.json").read_text())["weight_map"]
    omap = json.loads((outdir / "model.safetensors.index.json").read_text())["weight_map"]
    bad = []
    for key, shard in tmap.items():
        if key not in omap:
            bad.append((key, "missing-from-index"))
            continue
        te = read_st_header(template / shard)[0].get(key)
        oe = read_st_header(outdir / omap[key])[0].get(key)
        if oe is None:
            bad.append((key, "missing-in-shard"))
        elif te["dtype"] != oe["dtype"] or list(te["shape"]) != list(oe["shape"]):
            bad.append((key, f"{te['dtype']}{te['shape']} vs {oe['dtype']}{oe['shape']}"))
    return bad


def shards_identical(a, b) -> bool:
    """Every *.safetensors shard of directory a equals b's byte for byte."""
    import filecmp
    same = True
    for f in sorted(Path(a).glob("*.safetensors")):
        if not filecmp.cmp(f, Path(b) / f.name, shallow=False):
            same = False
    return same


def default_tmpdir(out) -> str:
    return os.environ.get("XTQ_TMPDIR") or str(Path(out).parent)

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

Assembly (the output of the reference's export_exl3.py:83-149): every
provided field is checked against its slot in the template's headers, then
each template shard is streamed to the output with those slots' bytes taken
from the fields (headers unchanged, so a template's own tensors written back
reproduce it byte for byte); every other file is copied as is and the
ARTIFACTS.sha256 manifest is rebuilt.

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
from dataclasses import dataclass
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


def tensor_info(module: str, result: dict, meta: dict | None = None) -> dict:
    """The .json metadata of one quantized tensor."""
    info = {"module": module, "K": int(result["K"]), "Wscale": float(result["Wscale"]),
            "code": result.get("code", "exl3_mul1"),
            "channel_scales": bool(result.get("channel_scales", False))}
    if meta:
        info.update(meta)
    return info


def save_fields(root, layer: int, module: str, fields: dict, info: dict) -> Path:
    """Write already-stored fields (stored_fields) and their metadata as
    ROOT/L{layer:02d}/{module}.safetensors + .json."""
    from safetensors.torch import save_file
    ldir = Path(root) / f"L{int(layer):02d}"
    ldir.mkdir(parents=True, exist_ok=True)
    path = ldir / f"{module}.safetensors"
    save_file(fields, str(path))
    path.with_suffix(".json").write_text(json.dumps(info, sort_keys=True))
    return path


def save_quantized(root, layer: int, module: str, result: dict,
                   meta: dict | None = None) -> Path:
    """Write ROOT/L{layer:02d}/{module}.safetensors (+ .json metadata) for one
    quantized tensor.  Returns the safetensors path."""
    return save_fields(root, layer, module, stored_fields(result),
                       tensor_info(module, result, meta))


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
@dataclass
class Blob:
    """One quantized field ready to be spliced into a template shard."""
    key: str                 # model.language_model.layers.{nn}.{module}.{field}
    tag: str                 # safetensors dtype tag, e.g. "I16"
    shape: list
    data: bytes


def _quant_files(tensors_root):
    """(layer index, module name, path) of every per-tensor file under
    ROOT/L*/, the module taken from the .json metadata when there is one."""
    for st_path in sorted(Path(tensors_root).glob("L*/*.safetensors")):
        layer = int(st_path.parent.name[1:])
        meta = st_path.with_suffix(".json")
        module = json.loads(meta.read_text()).get("module", st_path.stem) \
            if meta.exists() else st_path.stem
        yield layer, module, st_path


def collect_inputs(tensors_root) -> dict:
    """Every EXL3 field of the per-tensor files under ROOT, keyed by its name
    in the model: key -> (dtype tag, shape, raw little-endian bytes)."""
    from safetensors import safe_open
    blobs = {}
    for layer, module, path in _quant_files(tensors_root):
        with safe_open(str(path), framework="np") as f:
            names = set(f.keys())
            absent = [q for q in QUANT_FIELDS if q not in names]
            if absent:
                raise KeyError(f"{path} lacks the field(s) {absent}; it holds {sorted(names)}")
            for field in QUANT_FIELDS:
                arr = np.ascontiguousarray(f.get_tensor(field))
                tag = _ST_OF_NP.get(str(arr.dtype))
                if tag is None:
                    raise ValueError(f"{path}: field {field!r} is {arr.dtype}, which the "
                                     "EXL3 layout does not use")
                key = f"{LAYER_PREFIX}{layer}.{module}.{field}"
                blobs[key] = (tag, list(arr.shape), arr.tobytes())
    return blobs


def _plan_patches(blobs: dict, weight_map: dict, template: Path) -> dict:
    """shard name -> [(absolute byte offset, Blob)], every blob checked
    against the template's header entry before anything is written.  A blob
    must land on a tensor of the same dtype, shape and byte size."""
    plan: dict = {}
    headers: dict = {}
    for key, (tag, shape, data) in blobs.items():
        shard = weight_map.get(key)
        if shard is None:
            raise KeyError(f"{key}: not in template index -- the template model has no "
                           "tensor of that name")
        if shard not in headers:
            headers[shard] = read_st_header(template / shard)
        hdr, base = headers[shard]
        slot = hdr[key]
        if slot["dtype"] != tag or list(slot["shape"]) != list(shape):
            what = "dtype" if slot["dtype"] != tag else "shape"
            raise ValueError(f"{key}: {what} differs from the template's "
                             f"({tag} {list(shape)} produced, {slot['dtype']} "
                             f"{list(slot['shape'])} expected)")
        lo, hi = slot["data_offsets"]
        if hi - lo != len(data):
            raise ValueError(f"{key}: {len(data)} bytes produced, the template's slot "
                             f"holds {hi - lo}")
        plan.setdefault(shard, []).append((base + lo, Blob(key, tag, list(shape), data)))
    for patches in plan.values():
        patches.sort(key=lambda p: p[0])
    return plan


def _write_patched(src: Path, dst: Path, patches: list, chunk: int = 1 << 24) -> None:
    """Copy src to dst in one streaming pass, taking the bytes of each
    (offset, blob) patch from the blob instead of the source."""
    with open(src, "rb") as fi, open(dst, "wb") as fo:
        pos = 0
        for off, blob in patches + [(None, None)]:
            stop = off if off is not None else None
            while stop is None or pos < stop:
                want = chunk if stop is None else min(chunk, stop - pos)
                buf = fi.read(want)
                if not buf:
                    break
                fo.write(buf)
                pos += len(buf)
            if blob is not None:
                fo.write(blob.data)
                fi.seek(len(blob.data), os.SEEK_CUR)
                pos += len(blob.data)


def _write_manifest(outdir: Path) -> None:
    """ARTIFACTS.sha256: one "<sha256>  <name>" line per file of outdir."""
    entries = []
    for item in sorted(p for p in outdir.iterdir()
                       if p.is_file() and p.name != "ARTIFACTS.sha256"):
        digest = hashlib.sha256()
        with open(item, "rb") as f:
            for block in iter(lambda: f.read(1 << 24), b""):
                digest.update(block)
        entries.append(f"{digest.hexdigest()}  {item.name}")
    (outdir / "ARTIFACTS.sha256").write_text("\n".join(entries) + "\n")


def export(tensors_root, template, outdir) -> int:
    """Build a complete EXL3 model directory in OUTDIR from TEMPLATE with the
    quantized fields under TENSORS_ROOT spliced into the template's shards at
    their tensors' byte ranges (headers untouched, so the template's own
    tensors written back reproduce it byte for byte).  Every other template
    file is copied as is and the sha256 manifest is rebuilt.  All fields are
    validated before the first byte is written; returns how many were
    spliced."""
    template, outdir = Path(template), Path(outdir)
    weight_map = json.loads((template / "model.safetensors.index.json").read_text())["weight_map"]
    plan = _plan_patches(collect_inputs(tensors_root), weight_map, template)
    outdir.mkdir(parents=True, exist_ok=True)
    shards = set(weight_map.values())
    for shard in sorted(shards):
        _write_patched(template / shard, outdir / shard, plan.get(shard, []))
    for item in template.iterdir():
        if item.is_file() and item.name not in shards and item.name != "ARTIFACTS.sha256":
            shutil.copyfile(item, outdir / item.name)
    _write_manifest(outdir)
    return sum(len(p) for p in plan.values())


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

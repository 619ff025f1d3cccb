"""EXL3 writer and model-directory assembly (exl3b/export.py, the
export_exl3.py drop-in) on a synthetic template: byte-identical round trip
of the template's own tensors (the reference's --selftest-a), in-place
replacement, key / dtype / shape checks, fused mixed-K member layout."""
import json
import os
import subprocess
import sys

import pytest
import torch

from conftest import PKG

from exl3b import export as ex

MODULES = {0: [("self_attn.q_proj", 64, 96, 5), ("mlp.down_proj", 128, 64, 4)],
           1: [("self_attn.q_proj", 64, 96, 7), ("mlp.down_proj", 128, 64, 6)]}


def _fields(k, n, K, seed):
    g = torch.Generator().manual_seed(seed)
    return {
        "trellis": torch.randint(-32768, 32767, (k // 16, n // 16, 16 * K), generator=g,
                                 dtype=torch.int32).to(torch.int16),
        "suh": torch.randn(k, generator=g).half(),
        "svh": torch.randn(n, generator=g).half(),
    }


@pytest.fixture()
def template(tmp_path):
    """Two shards: layer 0 + embeddings in shard 1, layer 1 in shard 2."""
    from safetensors.torch import save_file
    tdir = tmp_path / "template"
    tdir.mkdir()
    wm = {}
    shard_t = {"model-00001-of-00002.safetensors": {}, "model-00002-of-00002.safetensors": {}}
    seed = 0
    for layer, mods in MODULES.items():
        shard = sorted(shard_t)[layer]
        for module, k, n, K in mods:
            seed += 1
            for field, t in _fields(k, n, K, seed).items():
                key = f"{ex.LAYER_PREFIX}{layer}.{module}.{field}"
                shard_t[shard][key] = t
                wm[key] = shard
    emb = "model.language_model.embed_tokens.weight"
    shard_t["model-00001-of-00002.safetensors"][emb] = torch.randn(32, 16).bfloat16()
    wm[emb] = "model-00001-of-00002.safetensors"
    for shard, tensors in shard_t.items():
        save_file(tensors, str(tdir / shard))
    (tdir / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))
    (tdir / "config.json").write_text(json.dumps({"quantization_config": {"bits": 5}}))
    (tdir / "ARTIFACTS.sha256").write_text("stale\n")
    return tdir


def test_selftest_a_byte_identical(template, tmp_path):
    root, n = ex.extract_template(template, tmp_path / "work")
    assert n == 4
    out = tmp_path / "out"
    assert ex.export(root, template, out) == 12
    assert ex.shards_identical(out, template)
    assert (out / "config.json").read_text() == (template / "config.json").read_text()
    lines = (out / "ARTIFACTS.sha256").read_text().split("\n")
    names = sorted(l.split()[1] for l in lines if l)
    assert names == sorted(p.name for p in out.iterdir() if p.name != "ARTIFACTS.sha256")
    assert ex.check_keys(template, out) == []


def test_export_replaces_blobs_in_place(template, tmp_path):
    root = tmp_path / "tensors"
    k, n, K = 128, 64, 6            # layer 1 down_proj is K=6 in the template
    g = torch.Generator().manual_seed(9)
    result = {"trellis": torch.randint(-3000, 3000, (k // 16, n // 16, 16 * K), generator=g,
                                       dtype=torch.int32).to(torch.int16),
              "suh": torch.where(torch.rand(k, generator=g) < 0.5, -1.0, 1.0).half(),
              "svh": torch.where(torch.rand(n, generator=g) < 0.5, -1.0, 1.0).half(),
              "Wscale": 0.0123, "K": K, "code": "exl3_mul1", "channel_scales": False}
    path = ex.save_quantized(root, 1, "mlp.down_proj", result)
    back = ex.load_quantized(path)
    assert back["meta"]["K"] == K and back["meta"]["module"] == "mlp.down_proj"
    # Wscale folded into suh (fp16), svh and trellis unchanged
    assert torch.equal(back["suh"], (result["suh"].float() * 0.0123).half())
    assert torch.equal(back["svh"], result["svh"]) and torch.equal(back["trellis"], result["trellis"])
    out = tmp_path / "out"
    assert ex.export(root, template, out) == 3
    base = f"{ex.LAYER_PREFIX}1.mlp.down_proj"
    wm = json.loads((template / "model.safetensors.index.json").read_text())["weight_map"]
    for field in ex.QUANT_FIELDS:
        got = ex.tensor_bytes(out / wm[f"{base}.{field}"], f"{base}.{field}")
        want = ex.stored_fields(result)[field].numpy().tobytes()
        assert got == want
    # untouched keys keep the template's bytes
    other = f"{ex.LAYER_PREFIX}0.mlp.down_proj.trellis"
    assert ex.tensor_bytes(out / wm[other], other) == ex.tensor_bytes(template / wm[other], other)
    assert ex.read_st_header(out / wm[other])[0] == ex.read_st_header(template / wm[other])[0]
    assert ex.check_keys(template, out) == []


def test_export_rejects_mismatches(template, tmp_path):
    root = tmp_path / "tensors"
    bad = {"trellis": torch.zeros(8, 4, 16 * 5, dtype=torch.int16), "suh": torch.ones(128).half(),
           "svh": torch.ones(64).half(), "Wscale": 1.0, "K": 5}
    ex.save_quantized(root, 0, "mlp.down_proj", bad)      # template has K=4 there
    with pytest.raises(ValueError, match="shape"):
        ex.export(root, template, tmp_path / "o1")
    root2 = tmp_path / "tensors2"
    ok = {"trellis": torch.zeros(8, 4, 64, dtype=torch.int16), "suh": torch.ones(128).half(),
          "svh": torch.ones(64).half(), "Wscale": 1.0, "K": 4}
    ex.save_quantized(root2, 7, "mlp.down_proj", ok)      # no layer 7 in the template
    with pytest.raises(KeyError, match="not in template"):
        ex.export(root2, template, tmp_path / "o2")


def test_fused_member_layout():
    k, ns, Ks = 64, [96, 32, 32], [5, 7, 7]
    offs = ex.fused_segments(k, ns, Ks)
    assert offs == [0, 4 * 6 * 80, 4 * 6 * 80 + 4 * 2 * 112, 4 * 6 * 80 + 2 * 4 * 2 * 112]
    trs = [_fields(k, n, K, 40 + j)["trellis"] for j, (n, K) in enumerate(zip(ns, Ks))]
    flat = ex.pack_fused(trs)
    assert flat.numel() == offs[-1]
    for a, b in zip(ex.unpack_fused(flat, k, ns, Ks), trs):
        assert torch.equal(a, b)
    with pytest.raises(ValueError):
        ex.unpack_fused(flat[:-1], k, ns, Ks)


def test_cli_selftest_a(template, tmp_path):
    r = subprocess.run([sys.executable, os.path.join(PKG, "export_exl3.py"), "--template",
                        str(template), "--out", str(tmp_path / "o"), "--selftest-a",
                        "--tmpdir", str(tmp_path)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "byte-identical: True" in r.stdout

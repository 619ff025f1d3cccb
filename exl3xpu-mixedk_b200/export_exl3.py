#!/usr/bin/env python3
"""Drop-in for the reference's ``quantize/export_exl3.py``: assemble a
complete EXL3 model directory from per-tensor trellis files.

    python export_exl3.py --tensors ROOT --template TEMPLATE_DIR --out OUT
        [--selftest-a] [--selftest-b L{nn}/{module}|W_hat.pt ...] [--check-keys]
        [--tmpdir DIR]

Input layout, scale convention and assembly rules: see exl3b/export.py.
--selftest-a  extract the template's own tensors, export them back and
              require byte-identical shards;
--selftest-b  dequantise written tensors on the GPU (weight_orig) and compare
              with a saved W_hat [out, in];
--check-keys  every template key present in the output with the same
              dtype / shape."""
import argparse
import os
import sys
import tempfile
from pathlib import Path

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from exl3b import export as ex  # noqa: E402


def selftest_b(outdir, specs):
    import json

    import torch
    from safetensors import safe_open
    wm = json.loads((Path(outdir) / "model.safetensors.index.json").read_text())["weight_map"]
    results = []
    for spec in specs:
        tensor_ref, wpath = spec.split("|")
        ldir, module = tensor_ref.split("/", 1)
        base = f"{ex.LAYER_PREFIX}{int(ldir[1:])}.{module}"
        with safe_open(str(Path(outdir) / wm[base + ".trellis"]), framework="pt") as f:
            trellis = f.get_tensor(base + ".trellis")
            suh = f.get_tensor(base + ".suh")
            svh = f.get_tensor(base + ".svh")
        K = trellis.shape[-1] // 16
        w = ex.weight_orig(trellis, suh, svh, K).t().contiguous().cpu()
        W_hat = torch.load(wpath, map_location="cpu", weights_only=False)
        results.append((tensor_ref, torch.equal(w, W_hat.contiguous()),
                        float((w - W_hat).abs().max())))
    return results


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tensors")
    ap.add_argument("--template", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--selftest-a", action="store_true")
    ap.add_argument("--selftest-b", nargs="*", default=None, metavar="L{nn}/{module}|W_hat.pt")
    ap.add_argument("--check-keys", action="store_true")
    ap.add_argument("--tmpdir", default=None)
    a = ap.parse_args()
    if a.selftest_a:
        parent = a.tmpdir or ex.default_tmpdir(a.out)
        Path(parent).mkdir(parents=True, exist_ok=True)
        with tempfile.TemporaryDirectory(dir=parent) as td:
            root, n = ex.extract_template(a.template, td)
            print(f"selftest-a: extracted {n} module(s) -> {root}")
            ex.export(root, a.template, a.out)
            same = ex.shards_identical(a.out, a.template)
            print(f"selftest-a: shards byte-identical: {same}")
            return 0 if same else 1
    if not a.tensors:
        ap.error("--tensors is required unless --selftest-a")
    n = ex.export(a.tensors, a.template, a.out)
    print(f"export: replaced {n} tensors -> {a.out}")
    rc = 0
    if a.selftest_b:
        for ref, eq, mx in selftest_b(a.out, a.selftest_b):
            print(f"selftest-b {ref}: equal={eq} maxabs={mx:.3e}")
            rc |= 0 if eq else 1
    if a.check_keys:
        bad = ex.check_keys(a.template, a.out)
        print(f"check-keys: {len(bad)} problems")
        for b in bad[:20]:
            print("  ", b)
        rc |= 1 if bad else 0
    return rc


if __name__ == "__main__":
    sys.exit(main())

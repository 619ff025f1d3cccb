"""The layer-stack driver on one GPU for part of one layer: the k/v members
of the attention fused module (K = 7 each under the SC5 table) share one
Hessian, are quantized in one sweep, and land as EXL3 files that dequantise
to the returned reconstruction."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_stack_layer_writes_members(tmp_path):
    from exl3b import export, stack, synth
    stats = stack.quantize_layer(0, torch.device("cuda", 0), out_root=tmp_path,
                                 tensors=["k", "v"])
    assert [(s["tensor"], s["K"]) for s in stats] == [("k", synth.SC5_K["k"]),
                                                      ("v", synth.SC5_K["v"])]
    for s in stats:
        f = export.load_quantized(tmp_path / "L00" / f"{stack.MODULE_NAMES[s['tensor']]}.safetensors")
        assert f["meta"]["K"] == s["K"] and f["meta"]["group"] == "attn"
        assert f["trellis"].shape == (5120 // 16, 1024 // 16, 16 * s["K"])
        assert s["Wscale"] > 0
        w = export.weight_orig(f["trellis"], f["suh"], f["svh"], s["K"]).t()
        W = synth.stack_weight(0, s["tensor"], "cuda").float()
        rel = float((w - W).square().sum() / W.square().sum())
        assert rel < 0.01, rel          # 7-bit trellis reconstruction error

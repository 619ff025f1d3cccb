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


def test_stack_hessian_files_and_writer_match_inline(tmp_path):
    """A Gram read from a dump file in the reference's naming gives the same
    EXL3 files as the synthetic one with the same values, written by the
    background writer instead of inline."""
    from safetensors.torch import save_file
    from exl3b import stack, synth
    dev = torch.device("cuda", 0)
    H = synth.hessian(5120, synth.stack_hessian_seed(0, "attn"), dev)
    hdir = tmp_path / "h"
    hdir.mkdir()
    save_file({"H": H.cpu()}, str(hdir / "L0_self_attn.q_proj.safetensors"))
    stack.quantize_layer(0, dev, out_root=tmp_path / "a", tensors=["k"])
    w = stack.Writer(tmp_path / "b")
    stats = stack.quantize_layer(0, dev, out_root=tmp_path / "b", tensors=["k"], writer=w,
                                 hessian_dir=hdir)
    w.close()
    assert stats[0]["synth_seconds"] >= 0 and stats[0]["seconds"] > 0
    for suffix in (".safetensors", ".json"):
        a = (tmp_path / "a" / "L00" / f"self_attn.k_proj{suffix}").read_bytes()
        b = (tmp_path / "b" / "L00" / f"self_attn.k_proj{suffix}").read_bytes()
        assert a == b, suffix


def test_harness_inputs_through_quantize():
    """quantize() on the harness inputs (check_tensor_bitexact.py:45-66:
    inner-domain weight and U with U^T U = G^-1) encodes the same problem as
    quantize_linear(W, H): with seed 128 and margin 0 the trellises agree
    except where the fp64 round trip of G through U moves a near tie."""
    from exl3b import api, harness
    gen = torch.Generator().manual_seed(17)
    k, n = 512, 256
    A = torch.randn(k, k, generator=gen)
    H = A.t() @ A / k + 0.1 * torch.eye(k)
    W = torch.randn(n, k, generator=gen) * 0.02
    Wt, U = harness.build_inputs(W, H)
    assert Wt.shape == (n, k) and U.shape == (k, k)
    assert torch.all(torch.tril(U, -1) == 0)
    W_hat, packed, scale = api.quantize(Wt, U, "exl3_mul1", 4, seed=128, margin=0)
    ref = api.quantize_linear(W, H, K=4, out_device="cuda")
    assert abs(scale - ref["Wscale"]) <= 1e-6 * ref["Wscale"]
    same = (packed == ref["trellis"]).all(-1).float().mean().item()
    assert same >= 0.9, same
    e_h = float((W_hat - Wt).square().sum() / Wt.square().sum())
    inner_ref = api.to_inner(ref["W_hat"].t(), ref["suh"].float(), ref["svh"].float())
    e_r = float((inner_ref.t() - Wt).square().sum() / Wt.square().sum())
    assert abs(e_h - e_r) <= 0.02 * e_r, (e_h, e_r)


def test_layer_split_one_rank_matches_layer_driver(tmp_path):
    """quantize_layer_split in a single process (a world of one: every
    tensor whole, through the column-range path with one LDL factor per
    input group) writes the same EXL3 fields as quantize_layer's fused
    modules, for a full layer of the stack at its mixed K."""
    from exl3b import export, stack, synth
    dev = torch.device("cuda", 0)
    stack.quantize_layer(0, dev, out_root=tmp_path / "a")
    stats = stack.quantize_layer_split(0, dev, out_root=tmp_path / "b")
    assert [s["tensor"] for s in stats] == [n for n, _o, _i in synth.STACK_SHAPES]
    for name, _o, _i in synth.STACK_SHAPES:
        a = export.load_quantized(tmp_path / "a" / "L00" / f"{stack.MODULE_NAMES[name]}.safetensors")
        b = export.load_quantized(tmp_path / "b" / "L00" / f"{stack.MODULE_NAMES[name]}.safetensors")
        for key in ("trellis", "suh", "svh"):
            assert torch.equal(a[key], b[key]), (name, key)
        assert a["meta"]["K"] == b["meta"]["K"] == synth.SC5_K[name]

"""The "blackhole-hex" vLLM quantization method (blackhole_b200.vllm_hex), the
drop-in for runtime/blackhole_runtime/vllm_hex.py: registration with the vLLM
in this image, the checkpoint-name mapping (vllm_hex.py:32, 104-115) and the
tier assembly and its refusals (vllm_hex.py:117-140), on CPU with a stand-in
layer.  The forward (apply) runs in the GPU test at the end."""

from __future__ import annotations

import types

import pytest
import torch

from blackhole_b200 import hex_data as hd

vllm = pytest.importorskip("vllm")

E, H, I, K = 12, 128, 64, 4


def _method():
    from blackhole_b200 import vllm_hex
    vllm_hex.register()
    return vllm_hex, vllm_hex._registered["moe"](types.SimpleNamespace(tp_size=1, ep_size=1))


def _checkpoint(seed=3):
    L = hd.synth_layer(E, H, I, "mixed", 32, seed=seed)
    out = []
    for t in L.tiers:
        pre = f"model.layers.0.mlp.experts.tier{1 << t['bits']}"
        out.append((f"{pre}.experts", t["experts"].to(torch.int32)))
        for p in ("gate_proj", "up_proj", "down_proj"):
            for q in ("idx", "block_scale", "expert_scale", "levels"):
                out.append((f"{pre}.{p}.{q}", t[p][q]))
    return L, out


def _layer(method, weights):
    layer = torch.nn.Module()
    layer.layer_name = "model.layers.0.mlp.experts"
    method.create_weights(layer, E, H, I, torch.bfloat16)
    loaded = list(layer.load_weights(iter(weights)))
    return layer, loaded


def test_registered_with_vllm():
    from vllm.model_executor.layers.quantization import QUANTIZATION_METHODS, get_quantization_config
    vh, _ = _method()
    assert vh.NAME in QUANTIZATION_METHODS
    cfg_cls = get_quantization_config(vh.NAME)
    cfg = cfg_cls.from_config({"quant_method": vh.NAME, "version": 1, "block": 32})
    assert cfg.get_name() == vh.NAME and cfg.get_min_capability() == 100
    assert cfg.get_supported_act_dtypes() == [torch.bfloat16, torch.float16]
    vh.register()                                   # idempotent


def test_trimmed_head_matches_full_head_on_kept_ids():
    """The output-trimmed LM head (HexHeadMethod, for a config with head_ids):
    kept logits equal the full head's, every other logit is HEAD_FILL."""
    vh, _ = _method()
    V, D = 50, 16
    g = torch.Generator().manual_seed(4)
    layer = torch.nn.Module()
    layer.weight = torch.nn.Parameter(torch.randn(V, D, generator=g), requires_grad=False)
    keep = [3, 7, 7, 41, 0]
    head = vh._registered["head"](keep)
    head.process_weights_after_loading(layer)
    x = torch.randn(5, D, generator=g)
    bias = torch.randn(V, generator=g)
    for b in (None, bias):
        got = head.apply(layer, x, b)
        full = torch.nn.functional.linear(x, layer.weight, b)
        kept = sorted(set(keep))
        assert got.shape == full.shape
        assert torch.allclose(got[:, kept], full[:, kept], rtol=1e-5, atol=1e-5)
        mask = torch.ones(V, dtype=torch.bool)
        mask[kept] = False
        assert bool((got[:, mask] == vh.HEAD_FILL).all())
    with pytest.raises(ValueError):
        vh._registered["head"]([V]).process_weights_after_loading(layer)


def test_names_load_into_tiers():
    vh, m = _method()
    L, ck = _checkpoint()
    layer, loaded = _layer(m, ck)
    assert sorted(loaded) == sorted(vh.param_name(n) for n, _ in ck)
    m.process_weights_after_loading(layer)
    assert [t.bits for t in layer.hex_tiers] == [4, 3]
    got = {int(e): t.bits for t in layer.hex_tiers for e in t.experts}
    want = {int(e): t["bits"] for t in L.tiers for e in t["experts"]}
    assert got == want


def test_refusals():
    vh, m = _method()
    with pytest.raises(ValueError, match="one GPU"):
        vh._registered["moe"](types.SimpleNamespace(tp_size=2, ep_size=1)).create_weights(
            torch.nn.Module(), E, H, I, torch.bfloat16)
    _, ck = _checkpoint()
    with pytest.raises(ValueError, match="unexpected expert tensor"):
        _layer(m, ck + [("model.layers.0.mlp.experts.w13_weight", torch.zeros(1))])
    layer, _ = _layer(m, [(n, t) for n, t in ck if "tier8" not in n])      # the 3-bit experts never arrive
    with pytest.raises(ValueError, match="no weights for experts"):
        m.process_weights_after_loading(layer)
    layer, _ = _layer(m, [(n, t) for n, t in ck if not n.endswith("tier16.up_proj.levels")])
    with pytest.raises(ValueError, match="missing"):
        m.process_weights_after_loading(layer)


@pytest.mark.gpu
def test_apply_matches_hex_moe():
    from blackhole_b200.hex_moe import hex_moe
    vh, m = _method()
    _, ck = _checkpoint(seed=9)
    torch.cuda.set_device(0)
    layer, _ = _layer(m, ck)
    m.process_weights_after_loading(layer)
    dev = torch.device("cuda", 0)
    w, ids = hd.synth_routing(40, E, K, seed=4, device=dev)
    x = hd.synth_x(40, H, seed=5, device=dev)
    got = m.apply(layer, x, w, ids.to(torch.int32), None, None)
    want = hex_moe(x, w, ids, layer.hex_tiers)
    assert torch.equal(got, want)

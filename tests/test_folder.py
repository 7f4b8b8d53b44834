"""blackhole-hex folders (blackhole_b200.folder): the tensor-name contract of the
reference's plugin and checker (runtime/blackhole_runtime/vllm_hex.py:32,
check_folder.py:22-44), read back bit for bit, and the structural checks of
check_folder.py:47-71.  The kernel half of the check runs in the GPU test at the
end of this file."""

from __future__ import annotations

import json

import pytest
import torch

from blackhole_b200 import hex_data as hd
from blackhole_b200.folder import check_folder, layer_tiers, read_tiers, save_folder

E, H, I, K = 12, 128, 64, 4
PRE = ("model.layers.{}.mlp.experts")


def _write(tmp_path, n_layers=2, bits="mixed", device="cpu"):
    layers = {PRE.format(i): hd.synth_layer(E, H, I, bits, 32, seed=30 + i, device=device).tiers
              for i in range(n_layers)}
    cfg = {"architectures": ["SyntheticMoe"], "num_experts": E, "num_experts_per_tok": K, "hidden_size": H,
           "moe_intermediate_size": I}
    save_folder(tmp_path, layers, cfg, shard_bytes=64 << 10)     # several shards
    return layers


def test_save_read_round_trip(tmp_path):
    layers = _write(tmp_path)
    assert len(list(tmp_path.glob("*.safetensors"))) > 1
    assert json.loads((tmp_path / "config.json").read_text())["quantization_config"]["quant_method"] == "blackhole-hex"
    got = read_tiers(tmp_path)
    assert sorted(got) == sorted(layers)
    for pre, tiers in layers.items():
        assert sorted(got[pre]) == sorted(1 << t["bits"] for t in tiers)
        for t in tiers:
            g = got[pre][1 << t["bits"]]
            assert torch.equal(g["experts"], t["experts"].to(torch.int32))
            for p in ("gate_proj", "up_proj", "down_proj"):
                for q in ("idx", "block_scale", "expert_scale", "levels"):
                    assert torch.equal(g[p][q], t[p][q]), (pre, p, q)


def test_layer_tiers_are_prepared_16_levels_first(tmp_path):
    _write(tmp_path, n_layers=1)
    tiers = layer_tiers(read_tiers(tmp_path)[PRE.format(0)], E, "cpu")
    assert [t.bits for t in tiers] == [4, 3]
    assert tiers[0].lookup is not None and tiers[0].dims() == (I, H)
    held = torch.cat([t.experts for t in tiers]).sort().values
    assert held.tolist() == list(range(E))


def test_structural_checks(tmp_path):
    _write(tmp_path)
    r = check_folder(tmp_path, run_kernel=False)
    assert r["ok"] and r["layers"] == 2 and r["checked"] == 0, r

    # an expert held twice (and another by none)
    from safetensors.torch import load_file, save_file
    f = sorted(tmp_path.glob("*.safetensors"))
    name = next(n for fp in f for n in load_file(str(fp)) if n.endswith(".experts") and PRE.format(1) in n)
    for fp in f:
        d = load_file(str(fp))
        if name in d:
            d[name] = d[name].clone()
            d[name][0] = d[name][1]
            save_file(d, str(fp), metadata={"format": "pt"})
    r = check_folder(tmp_path, run_kernel=False)
    assert not r["ok"] and any("exactly once" in p for p in r["problems"]), r

    cfg = json.loads((tmp_path / "config.json").read_text())
    cfg["quantization_config"]["quant_method"] = "fp8"
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    r = check_folder(tmp_path, run_kernel=False)
    assert any("not 'blackhole-hex'" in p for p in r["problems"]), r


def test_missing_part_is_reported(tmp_path):
    _write(tmp_path, n_layers=1)
    from safetensors.torch import load_file, save_file
    for fp in tmp_path.glob("*.safetensors"):
        d = load_file(str(fp))
        d = {n: v for n, v in d.items() if not n.endswith("tier8.down_proj.levels")}
        save_file(d, str(fp), metadata={"format": "pt"})
    r = check_folder(tmp_path, run_kernel=False)
    assert any("missing down_proj.levels" in p for p in r["problems"]), r


def test_command_line_structural_check(tmp_path, capsys):
    from blackhole_b200.folder import main
    _write(tmp_path, n_layers=1)
    assert main([str(tmp_path), "--no-kernel"]) == 0
    r = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert r["ok"] and r["layers"] == 1
    (tmp_path / "config.json").write_text(json.dumps({"quantization_config": {"quant_method": "awq"}}))
    assert main([str(tmp_path), "--no-kernel"]) == 1


@pytest.mark.gpu
def test_check_folder_runs_the_kernel(tmp_path):
    _write(tmp_path)
    r = check_folder(tmp_path, device="cuda")
    assert r["ok"] and r["checked"] == 2 and r["kernel_rel"] < 2e-2, r


@pytest.mark.parametrize("bits,block", [("3", 32), ("4", 128), ("mixed", 32)])
def test_checker_arithmetic_matches_oracle(oracle, bits, block):
    """The folder check's own reference (format_dequant, reference_moe) equals
    the pinned oracle: dequantization bit for bit, the layer within 1e-5."""
    import numpy as np
    from helpers import np_tiers

    from blackhole_b200.folder import format_dequant, reference_moe
    Hq, Iq = 256, 128          # multiples of the 128-input scale block
    L = hd.synth_layer(E, Hq, Iq, bits, block, seed=70)
    for t, nt in zip(L.tiers, np_tiers(L.tiers)):
        ex = torch.arange(len(t["experts"]))
        for p in ("gate_proj", "up_proj", "down_proj"):
            got = format_dequant(t[p], t["bits"], ex).numpy()
            want = oracle.dequant(nt[p], t["bits"], block)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), p
    w, ids = hd.synth_routing(9, E, K, seed=71)
    x = hd.synth_x(9, Hq, seed=72)
    tiers = {1 << t["bits"]: t for t in L.tiers}
    got = reference_moe(x, w, ids, tiers).numpy()
    want = oracle.moe_reference(x.float().numpy(), w.numpy(), ids.numpy(), np_tiers(L.tiers), E, block=block)
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()

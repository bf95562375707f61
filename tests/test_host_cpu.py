"""CPU-only tests: C-ABI surface, precision dispatch, bank accounting, install
validation and graph-replay host logic.  No GPU compute is invoked.

Mirrors the reference's own CPU tests where they exist (tests/test_method.py
BankTests: bank validation, storage audit, ContextVar non-leakage)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from actune_b200 import _lib
from actune_b200.layers import expected_version_bytes, install_bank, tensor_storage_bytes
from actune_b200.precision import (CONFIGURATIONS, SharedBank, active_precision_profile, pair,
                                   precision_profile)

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols(header):
    text = (ROOT / "include" / header).read_text()
    decl = r"^\s*(?:int|size_t|const char\s*\*)\s+(actune_[a-z0-9_]+)\s*\("
    return sorted(set(re.findall(decl, text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(str(_lib.LIB_PATH))
    for header in ("actune_b200.h", "actune_b200_harness.h"):
        for name in declared_symbols(header):
            assert hasattr(L, name), f"{name} declared in {header} but not exported"
    assert set(_lib.EXPORTS) <= set(declared_symbols("actune_b200.h"))


def test_abi_version_and_status_strings():
    L = _lib.lib()
    assert L.actune_abi_version() == 1
    for code in range(6):
        assert _lib.status_string(code)
    assert "unknown" in _lib.status_string(99)


def test_abi_rejects_bad_arguments_before_touching_a_device():
    L = _lib.lib()
    null = ctypes.c_void_p(0)
    # W outside {2,4,8}, K not a multiple of 64, negative M: rejected by validation.
    assert L.actune_packed_linear(null, null, null, null, null, 0, null, 3, 4, 4, 64, 3, 8, 0, null) == 1
    assert L.actune_packed_linear(null, null, null, null, null, 0, null, 3, 4, 4, 63, 4, 8, 0, null) == 1
    assert L.actune_packed_linear(null, null, null, null, null, 0, null, 3, -1, 4, 64, 4, 8, 0, null) == 1
    assert L.actune_quantize_group64(null, 3, 4, 64, 5, null, null, null) == 1
    assert L.actune_quantize_group64(null, 7, 4, 64, 8, null, null, null) == 1
    assert L.actune_pack_rows(null, 4, 63, 2, null, null) == 1
    assert L.actune_grouped_linear_workspace_size(600, 4096, 8) == 600 * 4096 + 600 * 64 * 4
    assert L.actune_grouped_linear_workspace_size(0, 4096, 8) == 0


def test_precision_profile_is_request_scoped():
    assert active_precision_profile() is None
    with precision_profile("q00"):
        with precision_profile("q11"):
            assert active_precision_profile() == "q11"
        assert active_precision_profile() == "q00"
    assert active_precision_profile() is None
    with pytest.raises(ValueError, match="Unknown"):
        with precision_profile("q22"):
            pass


def test_pair_parses_the_nine_modes():
    assert pair("w4a8") == (4, 8)
    assert sorted(pair(f"w{w}a{a}") for w in (2, 4, 8) for a in (2, 4, 8)) == [
        (w, a) for w in (2, 4, 8) for a in (2, 4, 8)]
    with pytest.raises(ValueError):
        pair("w3a8")


def bank_fixture(budget="w4a8"):
    shapes = {f"layer{i}": [8, 128] for i in range(8)}
    counts = {n: 128 for n in shapes}
    low = "w2a8" if budget == "w4a8" else "w2a4"
    base = "w4a8" if budget == "w4a8" else "w4a4"
    configs = {"q11": {n: base for n in shapes}}
    configs["q10"] = {**configs["q11"], "layer1": low}
    configs["q01"] = {**configs["q11"], "layer0": low}
    configs["q00"] = {**configs["q11"], "layer0": low, "layer1": low}
    sizes = {n: {m: expected_version_bytes(8, 128, int(m[1]), int(m[3])) for m in (base, low)} for n in shapes}
    return SharedBank(configs, shapes, counts, [list(shapes)], sizes, budget, 10 ** 6)


@pytest.mark.parametrize("budget", ["w4a8", "w4a4"])
def test_bank_validates_and_shares_alternatives(budget):
    bank = bank_fixture(budget).validate()
    full = sum(sum(bank.version_bytes[n][m] for n, m in c.items()) for c in bank.configurations.values())
    assert bank.resident_bytes() < full
    assert len({tuple(c.values()) for c in bank.configurations.values()}) == 4
    for q in CONFIGURATIONS:
        m = bank.check_request(q)
        assert m["weight_bits"] <= 4


def test_bank_rejections():
    bank = bank_fixture()
    bank.storage_limit = bank.resident_bytes() - 1
    with pytest.raises(ValueError, match="resident"):
        bank.validate()
    with pytest.raises(ValueError, match="target"):
        bank.check_request("q11", {})
    bank = bank_fixture()
    bank.configurations["q00"] = dict(bank.configurations["q11"])
    with pytest.raises(ValueError):
        bank.validate()
    bank = bank_fixture()
    bank.configurations["q11"]["layer3"] = "w8a8"  # a third switchable matrix, weight budget > 4
    with pytest.raises(ValueError):
        bank.validate()


def test_install_bank_checks_targets_before_touching_the_model():
    bank = bank_fixture()
    model = torch.nn.Module()
    for i in range(8):
        setattr(model, f"layer{i}", torch.nn.Linear(128, 8, bias=False))
    model.layer3 = torch.nn.Linear(128, 9, bias=False)  # wrong shape
    with pytest.raises(ValueError, match="calibrated matrix: layer3"):
        install_bank(model, bank, {n: {} for n in bank.shapes})
    assert isinstance(model.layer0, torch.nn.Linear)  # untouched


def test_expected_version_bytes_matches_buffer_layout():
    # packed [N, Kpad*W/8] uint8 + f32 [N] scale (+ bias: layer dtype, f32 when a == 4)
    assert expected_version_bytes(4096, 4096, 4, 8) == 4096 * 2048 + 4 * 4096
    assert expected_version_bytes(96, 100, 2, 8) == 96 * 128 // 4 + 4 * 96
    assert expected_version_bytes(96, 128, 8, 4, torch.bfloat16) == 96 * 128 + 4 * 96 + 4 * 96
    assert expected_version_bytes(96, 128, 8, 8, torch.bfloat16) == 96 * 128 + 4 * 96 + 2 * 96
    m = torch.nn.Module()
    m.register_buffer("a", torch.zeros(10, dtype=torch.uint8))
    m.register_buffer("b", torch.zeros(3, dtype=torch.float32))
    assert tensor_storage_bytes(m) == 10 + 12


def test_graph_replay_disabled_is_a_passthrough():
    from actune_b200.graph import GraphReplay
    calls = []

    def fn(x):
        calls.append(x)
        return x + 1

    g = GraphReplay(fn, {}, max_graphs=2)
    assert g(3) == 4 and calls == [3] and g.replays == 0


def test_graph_replay_key_depends_on_shape_and_precision():
    from actune_b200.graph import GraphReplay

    class Layer:
        def __init__(self, assignments):
            self.assignments, self.default_profile = assignments, "q11"
            self.calls = self.input_elements = 0

    layers = {"a": Layer({"q00": "w2a8", "q01": "w2a8", "q10": "w4a8", "q11": "w4a8"})}
    g = GraphReplay(lambda x: x, layers)
    from torch.utils import _pytree as pytree
    leaves, tree = pytree.tree_flatten(((torch.zeros(2, 3),), {}))
    k_default = g.key(leaves, tree)
    with precision_profile("q00"):
        k00 = g.key(leaves, tree)
    with precision_profile("q11"):
        k11 = g.key(leaves, tree)
    assert k_default == k11 and k00 != k11
    leaves2, tree2 = pytree.tree_flatten(((torch.zeros(4, 3),), {}))
    assert g.key(leaves2, tree2) != k_default


def test_shared_activation_scope_is_scoped():
    from actune_b200.kernels.grouped import _SHARED, shared_activation_scope
    assert _SHARED.get() is None
    with shared_activation_scope(True):
        assert _SHARED.get() == []
        with shared_activation_scope(False):
            assert _SHARED.get() is None
    assert _SHARED.get() is None


def test_forward_refuses_cpu_input():
    from actune_b200.kernels.grouped import GroupedLinear
    layer = GroupedLinear.__new__(GroupedLinear)
    torch.nn.Module.__init__(layer)
    layer.in_features, layer.out_features, layer.w, layer.a = 64, 8, 4, 8
    with pytest.raises(ValueError, match="requires CUDA"):
        layer(torch.zeros(2, 64))


def test_grouped_linear_rejects_bad_widths_and_k():
    from actune_b200.kernels.grouped import GroupedLinear
    with pytest.raises(ValueError, match="divisible by 64"):
        GroupedLinear(torch.nn.Linear(100, 8), 4, 8, None)
    with pytest.raises(ValueError, match="integer width"):
        GroupedLinear(torch.nn.Linear(128, 8), 3, 8, None)


def test_clip_ratio_validation_messages():
    from actune_b200.kernels.quantizers import _validate_clip_ratios
    assert _validate_clip_ratios(0.9, out_features=4, device="cpu").shape == (4,)
    with pytest.raises(ValueError, match="expected 4"):
        _validate_clip_ratios([0.5, 0.5], out_features=4, device="cpu")
    with pytest.raises(ValueError, match="finite"):
        _validate_clip_ratios(float("nan"), out_features=4, device="cpu")
    with pytest.raises(ValueError, match=r"\(0, 1\]"):
        _validate_clip_ratios(1.5, out_features=4, device="cpu")


def test_sweep_table_and_workload():
    """The config-1 sweep covers the 4 Llama-2-7B projection shapes and formats one
    markdown row per case (no GPU needed to check the host side)."""
    from actune_b200 import sweep
    assert sweep.SHAPES == {"qkv": (4096, 12288), "o": (4096, 4096), "gate_up": (4096, 22016),
                            "down": (11008, 4096)}
    row = {"W": 4, "A": 8, "shape": "qkv", "M": 1, "K": 4096, "N": 12288, "us": 14.5, "GBps": 1740.0,
           "hbm_frac": 0.27, "TOPS": 6.9, "int8_frac": 0.002}
    text = sweep.markdown({"hbm_gbs": 6456.8, "int8_tops": 3021.0, "rows": [row]})
    assert "| W4A8 | qkv | 1 | 14.5 | 1740.0 | 0.27 | 6.9 | 0.002 |" in text


def test_reference_arms_of_configs_0_and_1_report_unavailable_without_gpu_work(monkeypatch, capsys):
    """bench.py --impl reference: config 1 times the reference's own CUDA kernel built
    into oracle/_ref and prints one `unavailable` line when that module is absent;
    config 0 (W4A8, which the reference runs on its Triton kernel) always prints one.
    Neither touches a GPU on those paths."""
    import json
    import sys
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    import bench
    from oracle import build_ref
    monkeypatch.setattr(build_ref, "load", lambda name: None)
    monkeypatch.setattr(sys, "argv", ["bench.py", "--impl", "reference", "--config", "1"])
    bench.main()
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "oracle/_ref" in line["unavailable"]
    monkeypatch.setattr(sys, "argv", ["bench.py", "--impl", "reference", "--config", "0"])
    bench.main()
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "Triton" in line["unavailable"]

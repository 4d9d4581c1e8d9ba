"""Knob registry (override > environment > default, typed parsing, the
startup table) and YAML / JSON run configs (typed sections, unknown keys
rejected, CLI flags over file values)."""
import json

import pytest

from rlx_models_b200 import settings


@pytest.fixture(autouse=True)
def _clean(monkeypatch):
    for name in settings.KNOBS:
        monkeypatch.delenv(name, raising=False)
    settings.clear_overrides()
    yield
    settings.clear_overrides()


def test_knob_precedence(monkeypatch):
    assert settings.get("B200_TP_TWO_SHOT") == "auto" and settings.source("B200_TP_TWO_SHOT") == "default"
    monkeypatch.setenv("B200_TP_TWO_SHOT", "off")
    assert settings.get("B200_TP_TWO_SHOT") == "off" and settings.source("B200_TP_TWO_SHOT") == "env"
    settings.override("B200_TP_TWO_SHOT", "on")
    assert settings.get("B200_TP_TWO_SHOT") == "on" and settings.source("B200_TP_TWO_SHOT") == "override"
    import os
    assert os.environ["B200_TP_TWO_SHOT"] == "on"  # exported for readers of the environment
    monkeypatch.setenv("B200_PDL", "0")
    assert settings.get("B200_PDL") is False
    with pytest.raises(ValueError):
        settings.override("B200_TP_TWO_SHOT", "sometimes")
    with pytest.raises(KeyError):
        settings.override("B200_NOT_A_KNOB", 1)


def test_describe_lists_every_knob():
    t = settings.describe()
    for name in settings.KNOBS:
        assert name in t


def test_every_knob_in_the_code_is_declared():
    """Each B200_* / RLX_* environment switch read anywhere in the package is in the registry."""
    import os
    import re
    root = os.path.dirname(settings.__file__)
    found = set()
    for d, _, files in os.walk(root):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")) and f != "settings.py":
                txt = open(os.path.join(d, f), errors="ignore").read()
                found |= set(re.findall(r'(?:getenv|environ\.get|settings\.get)\(\s*"((?:RLX_)?B200_[A-Z0-9_]+)"', txt))
    assert found, "no knob reads found"
    assert found <= set(settings.KNOBS), sorted(found - set(settings.KNOBS))


def test_run_config_yaml_and_json(tmp_path):
    y = tmp_path / "run.yaml"
    y.write_text("model: qwen3-0.6b\nparallel: {tp: 2, tp_comm: nccl}\n"
                 "serve: {max_num_seqs: 12, kv_memory_gb: 2.5, graph_batch_sizes: [1, 2, 4]}\n"
                 "train: {lr: 3.0e-4, optimizer: muon, betas: [0.9, 0.99]}\nkernel: {B200_PDL: 0}\n")
    rc = settings.load_run_config(str(y))
    assert rc.model == "qwen3-0.6b" and rc.parallel.tp == 2 and rc.parallel.world() == 2
    ec = rc.engine_config(max_model_len=777)
    assert ec.max_num_seqs == 12 and ec.kv_memory_gb == 2.5 and ec.max_model_len == 777
    assert ec.graph_batch_sizes == (1, 2, 4)
    tc = rc.train_config()
    assert tc.lr == 3e-4 and tc.optimizer == "muon" and tc.betas == (0.9, 0.99)
    rc.apply_kernel_overrides()
    assert settings.get("B200_PDL") is False
    j = tmp_path / "run.json"
    j.write_text(json.dumps({"serve": {"max_num_seqs": 3}}))
    assert settings.load_run_config(str(j)).engine_config().max_num_seqs == 3


@pytest.mark.parametrize("bad", [{"serve": {"max_seqs": 1}}, {"paralel": {}}, {"kernel": {"B200_NOPE": 1}},
                                 {"parallel": {"tq": 2}}, {"kernel": {"B200_TP_TWO_SHOT": "maybe"}}])
def test_run_config_rejects_unknown_keys(tmp_path, bad):
    j = tmp_path / "bad.json"
    j.write_text(json.dumps(bad))
    with pytest.raises(ValueError):
        settings.load_run_config(str(j))


def test_cli_knobs_and_config(tmp_path, capsys):
    from rlx_models_b200.__main__ import main
    y = tmp_path / "k.yaml"
    y.write_text("kernel: {B200_NVTX: 1}\n")
    assert main(["knobs", "--config", str(y)]) == 0
    out = capsys.readouterr().out
    line = next(ln for ln in out.splitlines() if ln.startswith("B200_NVTX"))
    assert "True" in line and "override" in line

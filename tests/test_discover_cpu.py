"""Weight discovery over other tools' caches (LM Studio, Ollama, HF hub, extra
roots) in temporary directories: formats recognised, Ollama manifests mapped
to their GGUF blobs, queries resolved with quantisation and source preference."""
import json
import os
import struct

from rlx_models_b200.weights import discover as D


def _gguf(path):
    os.makedirs(os.path.dirname(path), exist_ok=True)
    with open(path, "wb") as f:
        f.write(b"GGUF" + struct.pack("<IQQ", 3, 0, 0))


def test_scan_and_resolve(tmp_path):
    lms = tmp_path / "lms"
    _gguf(str(lms / "Qwen" / "Qwen3-0.6B-GGUF" / "Qwen3-0.6B-Q8_0.gguf"))
    _gguf(str(lms / "Qwen" / "Qwen3-0.6B-GGUF" / "Qwen3-0.6B-Q4_K_M.gguf"))
    with open(lms / "Qwen" / "not-a-model.gguf", "wb") as f:  # wrong magic: ignored
        f.write(b"JUNK")
    oll = tmp_path / "ollama"
    man = oll / "manifests" / "registry.ollama.ai" / "library" / "qwen2.5"
    man.mkdir(parents=True)
    _gguf(str(oll / "blobs" / "sha256-deadbeef"))
    (man / "32b").write_text(json.dumps({"layers": [{"digest": "sha256:deadbeef",
                                                      "mediaType": "application/vnd.ollama.image.model"}]}))
    hf = tmp_path / "hub"
    snap = hf / "models--org--Cool-Model" / "snapshots" / "abc"
    snap.mkdir(parents=True)
    (snap / "config.json").write_text("{}")
    (snap / "model.safetensors").write_bytes(b"\0" * 8)
    roots = [("lmstudio", str(lms)), ("ollama", str(oll)), ("hf", str(hf))]
    hits = D.scan(roots)
    names = sorted(h.name for h in hits)
    assert "ollama:qwen2.5:32b" in names and "org/Cool-Model" in names
    assert sum(h.fmt == "gguf" for h in hits) == 3
    assert D.resolve("qwen3-0.6b", roots).endswith("Qwen3-0.6B-Q4_K_M.gguf")
    assert D.resolve("qwen3-0.6b", roots, prefer_quant="Q8_0").endswith("Q8_0.gguf")
    assert D.resolve("ollama:qwen2.5:32b", roots) == str(oll / "blobs" / "sha256-deadbeef")
    assert D.resolve("org/cool-model", roots) == str(snap)
    assert D.resolve("missing", roots) is None


def test_env_roots(tmp_path, monkeypatch):
    monkeypatch.setenv("RLX_WEIGHTS_PATHS", str(tmp_path / "a") + os.pathsep + str(tmp_path / "b"))
    monkeypatch.setenv("OLLAMA_MODELS", str(tmp_path / "o"))
    roots = D.default_roots()
    assert ("extra", str(tmp_path / "b")) in roots and ("ollama", str(tmp_path / "o")) in roots

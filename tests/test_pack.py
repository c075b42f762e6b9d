"""Pack host logic: config validation, manifest verification and the strict
safetensors parser, mirroring native/model_test.go:479-567 (tampered packs
fail loudly), native/safetensors_test.go and native/config.go:119-171."""
from __future__ import annotations

import json
import shutil
import struct

import numpy as np
import pytest

from conftest import GOLDEN
from futon_b200 import synth
from futon_b200.pack import (PackError, expected_tensor_shapes, load_pack,
                             load_pack_config, parse_safetensors, safetensors_bytes, sha256_file,
                             write_pack)

SRC = GOLDEN / "toy-absolute-gelu"


def copy_pack(tmp_path, src=SRC):
    dst = tmp_path / src.name
    shutil.copytree(src, dst)
    return dst


def mutate_json(path, fn):
    d = json.loads(path.read_text())
    fn(d)
    path.write_text(json.dumps(d))


def rehash_manifest(d):
    """Recomputes member hashes (not tensor_names), like rehashManifest."""
    def fix(m):
        for name in m["members"]:
            m["members"][name] = {"sha256": sha256_file(d / name), "size": (d / name).stat().st_size}
    mutate_json(d / "manifest.json", fix)


def drop_tensor(d, name):
    t = parse_safetensors((d / "model.safetensors").read_bytes())
    del t[name]
    (d / "model.safetensors").write_bytes(safetensors_bytes(t))


def test_loads_toy_packs():
    for pack in ("toy-absolute-gelu", "toy-rope-swiglu"):
        p = load_pack(GOLDEN / pack)
        assert p.cfg.model_id == pack
        assert set(p.tensors) == set(p.manifest["tensor_names"])
        want = expected_tensor_shapes(p.cfg)
        for name, arr in p.tensors.items():
            assert tuple(arr.shape) == want[name]


def test_extra_tensor(tmp_path):
    d = copy_pack(tmp_path)
    mutate_json(d / "config.json", lambda m: m.update(num_layers=1))
    rehash_manifest(d)
    p = load_pack(d)  # the host loader accepts; the upload rejects leftovers
    extra = set(p.tensors) - set(expected_tensor_shapes(p.cfg))
    assert extra, "num_layers=1 must leave layer-1 tensors unexpected"


@pytest.mark.parametrize("field,value,match", [
    ("pack_format", 99, "unsupported pack_format"),
    ("pre_norm", True, "pre_norm"),
    ("position_encoding", "alibi", "unknown position_encoding"),
    ("activation", "relu", "unknown activation"),
    ("pooling", "max", "unknown pooling"),
    ("layer_norm_eps", 0, "layer_norm_eps"),
    ("num_heads", 5, "not divisible"),
    ("max_trained_positions", 2, "max_trained_positions"),
])
def test_config_rejects(tmp_path, field, value, match):
    d = copy_pack(tmp_path)
    mutate_json(d / "config.json", lambda m: m.update({field: value}))
    rehash_manifest(d)
    with pytest.raises(PackError, match=match):
        load_pack(d)


def test_rope_requires_theta():
    c = synth.arch("nomic")
    c.rope_theta = 0
    with pytest.raises(PackError, match="rope_theta"):
        c.validate()


def test_matryoshka_dims_checked():
    c = synth.arch("nomic")
    c.matryoshka.dims = [769]
    with pytest.raises(PackError, match="matryoshka dim"):
        c.validate()


def test_truncated_weights(tmp_path):
    d = copy_pack(tmp_path)
    raw = (d / "model.safetensors").read_bytes()
    (d / "model.safetensors").write_bytes(raw[:-100])
    with pytest.raises(PackError):
        load_pack(d)


def test_missing_manifest(tmp_path):
    d = copy_pack(tmp_path)
    (d / "manifest.json").unlink()
    with pytest.raises(PackError, match="manifest.json unreadable"):
        load_pack(d)


def test_edited_config_stale_manifest(tmp_path):
    d = copy_pack(tmp_path)
    mutate_json(d / "config.json", lambda m: m.update(normalize=False))
    with pytest.raises(PackError, match="sha256|bytes"):
        load_pack(d)


def test_removed_optional_tensor(tmp_path):
    d = copy_pack(tmp_path)
    drop_tensor(d, "layers.0.attn.qkv.bias")
    with pytest.raises(PackError):
        load_pack(d)


def test_removed_optional_tensor_rehashed_manifest(tmp_path):
    d = copy_pack(tmp_path)
    drop_tensor(d, "layers.0.attn.qkv.bias")
    rehash_manifest(d)
    with pytest.raises(PackError, match="tensor set drifted"):
        load_pack(d)


def test_mixed_pack_contents(tmp_path):
    d = copy_pack(tmp_path)
    mutate_json(d / "manifest.json", lambda m: m.update(model_id="other"))
    with pytest.raises(PackError, match="mixed pack contents"):
        load_pack(d)


# ---- safetensors strictness (safetensors.go:104-221) ------------------------
def _st(header: dict, data: bytes) -> bytes:
    hj = json.dumps(header).encode()
    return struct.pack("<Q", len(hj)) + hj + data


def test_safetensors_rejects():
    ok = np.arange(4, dtype=np.float32).tobytes()
    parse_safetensors(_st({"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, ok))
    cases = [
        (_st({"a": {"dtype": "BF16", "shape": [4], "data_offsets": [0, 8]}}, ok[:8]), "unsupported dtype"),
        (_st({"a": {"dtype": "F32", "shape": [3], "data_offsets": [0, 16]}}, ok), "needs 12 bytes"),
        (_st({"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, ok + b"xx"), "cover"),
        (_st({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
              "b": {"dtype": "F32", "shape": [2], "data_offsets": [4, 12]}}, ok[:12]), "overlap or gap"),
        (_st({"a": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 0]}}, b""), "negative dimension"),
        (_st({"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 32]}}, ok), "outside data"),
        (b"\x01\x02", "too small"),
        (struct.pack("<Q", 1 << 40), "exceeds limit"),
    ]
    for raw, match in cases:
        with pytest.raises(PackError, match=match):
            parse_safetensors(raw)


def test_f16_tensors_exact():
    vals = np.array([0.0, -0.0, 1.0, 65504.0, 6e-8, -2.5, np.inf], dtype=np.float16)
    raw = _st({"h": {"dtype": "F16", "shape": [7], "data_offsets": [0, 14]}}, vals.tobytes())
    t = parse_safetensors(raw, keep_f16=False)["h"]
    assert t.dtype == np.float32
    assert np.array_equal(t, vals.astype(np.float32))
    assert parse_safetensors(raw, keep_f16=True)["h"].dtype == np.float16


def test_write_pack_roundtrip(tmp_path):
    cfg = synth.arch("nomic")
    cfg.num_layers, cfg.vocab_size = 1, 1200
    w = synth.make_weights(cfg)
    assert not any(k.endswith(".bias") and "norm" not in k for k in w)  # nomic: no linear biases
    d = write_pack(tmp_path / "p", cfg, w, synth.synthetic_vocab(cfg))
    p = load_pack(d, keep_f16=False)
    assert p.cfg == load_pack_config(d)
    for k, v in w.items():
        assert np.array_equal(p.tensors[k], v)

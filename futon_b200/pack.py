"""Weight packs: config.json, manifest.json, model.safetensors, vocab.txt.

Host-side mirror of futon's pack loader, so the B200 path loads exactly the
packs the reference loads:
  PackConfig / Validate / EffectiveMaxSeqLen   native/config.go:54-171
  manifest sha256 + size + tensor-name set      native/manifest.go:46-104
  strict safetensors parser (F32/F16 only)      native/safetensors.go:104-221
Every failure raises PackError with a message in the reference's wording.
`write_pack` produces packs in the same format (used for synthetic packs).
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
import os
import struct
from pathlib import Path
from typing import Dict, List, Optional

import numpy as np

PACK_FORMAT_VERSION = 1
POS_ABSOLUTE, POS_ROPE = "absolute", "rope"
ACT_GELU, ACT_SWIGLU = "gelu", "swiglu"
POOL_MEAN, POOL_CLS = "mean", "cls"
MAX_HEADER_BYTES = 16 << 20
MANIFEST_MEMBERS = ("config.json", "model.safetensors", "vocab.txt")


class PackError(ValueError):
    """A pack failed validation (the reference returns an error, never panics)."""


@dataclasses.dataclass
class Matryoshka:
    layernorm: bool = False
    dims: List[int] = dataclasses.field(default_factory=list)


@dataclasses.dataclass
class PackConfig:
    """Architecture description of a pack (native/config.go:54-102)."""

    pack_format: int = PACK_FORMAT_VERSION
    model_id: str = ""
    hidden_size: int = 0
    num_layers: int = 0
    num_heads: int = 0
    intermediate_size: int = 0
    vocab_size: int = 0
    type_vocab_size: int = 0
    max_seq_len: int = 0
    layer_norm_eps: float = 0.0
    position_encoding: str = ""
    rope_theta: float = 0.0
    max_trained_positions: int = 0
    activation: str = ""
    pre_norm: bool = False
    pooling: str = ""
    normalize: bool = False
    matryoshka: Optional[Matryoshka] = None
    tokenizer: dict = dataclasses.field(default_factory=dict)
    prefixes: dict = dataclasses.field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: dict) -> "PackConfig":
        kw = {}
        for f in dataclasses.fields(cls):
            if f.name in d:
                kw[f.name] = d[f.name]
        m = d.get("matryoshka")
        if m is not None:
            kw["matryoshka"] = Matryoshka(layernorm=bool(m.get("layernorm", False)),
                                          dims=list(m.get("dims", []) or []))
        return cls(**kw)

    def to_dict(self) -> dict:
        d = dataclasses.asdict(self)
        if self.matryoshka is None:
            d.pop("matryoshka")
        for k in ("rope_theta", "max_trained_positions", "pre_norm", "prefixes"):
            if not d.get(k):
                d.pop(k, None)
        return d

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    def effective_max_seq_len(self) -> int:
        """max_seq_len clamped to the trained context (config.go:111-116)."""
        if 0 < self.max_trained_positions < self.max_seq_len:
            return self.max_trained_positions
        return self.max_seq_len

    def validate(self) -> None:
        """Internal consistency checks (config.go:119-171)."""
        mid = self.model_id
        if self.pack_format != PACK_FORMAT_VERSION:
            raise PackError(f"pack: unsupported pack_format {self.pack_format} "
                            f"(loader supports {PACK_FORMAT_VERSION})")
        if not mid:
            raise PackError("pack: model_id missing")
        if min(self.hidden_size, self.num_layers, self.num_heads, self.intermediate_size) <= 0:
            raise PackError(f"pack {mid}: non-positive architecture dimension")
        if self.hidden_size % self.num_heads:
            raise PackError(f"pack {mid}: hidden_size {self.hidden_size} not divisible by "
                            f"num_heads {self.num_heads}")
        if self.vocab_size <= 0 or self.max_seq_len <= 2:
            raise PackError(f"pack {mid}: invalid vocab_size/max_seq_len")
        if self.max_trained_positions < 0 or 0 < self.max_trained_positions <= 2:
            raise PackError(f"pack {mid}: invalid max_trained_positions {self.max_trained_positions}")
        if self.layer_norm_eps <= 0:
            raise PackError(f"pack {mid}: layer_norm_eps must be positive")
        if self.position_encoding == POS_ROPE:
            if self.rope_theta <= 0:
                raise PackError(f"pack {mid}: rope position encoding requires rope_theta > 0")
        elif self.position_encoding != POS_ABSOLUTE:
            raise PackError(f"pack {mid}: unknown position_encoding {self.position_encoding!r}")
        if self.activation not in (ACT_GELU, ACT_SWIGLU):
            raise PackError(f"pack {mid}: unknown activation {self.activation!r}")
        if self.pooling not in (POOL_MEAN, POOL_CLS):
            raise PackError(f"pack {mid}: unknown pooling {self.pooling!r}")
        if self.pre_norm:
            raise PackError(f"pack {mid}: pre_norm is declared but not yet implemented — "
                            "refusing to run the wrong architecture")
        if self.matryoshka is not None:
            for dim in self.matryoshka.dims:
                if dim <= 0 or dim > self.hidden_size:
                    raise PackError(f"pack {mid}: matryoshka dim {dim} outside "
                                    f"(0,{self.hidden_size}]")


def load_pack_config(pack_dir: os.PathLike) -> PackConfig:
    """Reads and validates <dir>/config.json (config.go:174-187)."""
    path = Path(pack_dir) / "config.json"
    try:
        raw = path.read_bytes()
    except OSError as e:
        raise PackError(f"pack: read config: {e}") from e
    try:
        cfg = PackConfig.from_dict(json.loads(raw))
    except (ValueError, TypeError) as e:
        raise PackError(f"pack: parse config: {e}") from e
    cfg.validate()
    return cfg


def sha256_file(path: os.PathLike) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def load_and_verify_manifest(pack_dir: os.PathLike) -> dict:
    """sha256 + size of every consumed member (manifest.go:46-78)."""
    d = Path(pack_dir)
    try:
        man = json.loads((d / "manifest.json").read_bytes())
    except OSError as e:
        raise PackError(f"pack {d}: manifest.json unreadable (refusing to load an "
                        f"unverifiable pack): {e}") from e
    except ValueError as e:
        raise PackError(f"pack {d}: manifest.json malformed: {e}") from e
    members = man.get("members") or {}
    for member in MANIFEST_MEMBERS:
        meta = members.get(member)
        if meta is None:
            raise PackError(f"pack {d}: manifest records no entry for {member}")
        p = d / member
        if not p.exists():
            raise PackError(f"pack {d}: member {member}: missing")
        size = p.stat().st_size
        if size != meta.get("size"):
            raise PackError(f"pack {d}: member {member} is {size} bytes, manifest records "
                            f"{meta.get('size')}")
        got = sha256_file(p)
        if got != meta.get("sha256"):
            raise PackError(f"pack {d}: member {member} sha256 {got} does not match manifest "
                            f"{meta.get('sha256')} (tampered or corrupt — rebuild the pack)")
    return man


def verify_tensor_names(man: dict, tensors: Dict[str, np.ndarray]) -> None:
    """Exact tensor-name set when recorded (manifest.go:84-104)."""
    names = man.get("tensor_names")
    if names is None:
        return
    got, want = sorted(tensors), sorted(names)
    if len(got) != len(want):
        raise PackError(f"pack {man.get('model_id')}: {len(got)} tensors on disk, manifest "
                        f"records {len(want)} — tensor set drifted")
    for g, w in zip(got, want):
        if g != w:
            raise PackError(f"pack {man.get('model_id')}: tensor set drifted from manifest "
                            f"(first difference: {g!r} vs recorded {w!r})")


def parse_safetensors(raw: bytes, keep_f16: bool = False) -> Dict[str, np.ndarray]:
    """Strict safetensors parser (safetensors.go:104-221): F32/F16 only, shapes
    must match byte spans, spans must tile the data section exactly."""
    if len(raw) < 8:
        raise PackError(f"safetensors: file too small ({len(raw)} bytes) for header length prefix")
    (hlen,) = struct.unpack("<Q", raw[:8])
    if hlen > MAX_HEADER_BYTES:
        raise PackError(f"safetensors: header length {hlen} exceeds limit {MAX_HEADER_BYTES}")
    if len(raw) < 8 + hlen:
        raise PackError(f"safetensors: declared header length {hlen} exceeds file size {len(raw)}")
    try:
        header = json.loads(raw[8:8 + hlen])
    except ValueError as e:
        raise PackError(f"safetensors: parse header JSON: {e}") from e
    data = memoryview(raw)[8 + hlen:]
    tensors: Dict[str, np.ndarray] = {}
    spans = []
    for name, entry in header.items():
        if name == "__metadata__":
            continue
        dtype = entry.get("dtype")
        if dtype == "F32":
            esz, npdt = 4, np.dtype("<f4")
        elif dtype == "F16":
            esz, npdt = 2, np.dtype("<f2")
        else:
            raise PackError(f"safetensors: tensor {name!r}: unsupported dtype {dtype!r} "
                            "(want F32 or F16)")
        shape = [int(x) for x in entry.get("shape", [])]
        elems = 1
        for dim in shape:
            if dim < 0:
                raise PackError(f"safetensors: tensor {name!r}: negative dimension {dim}")
            elems *= dim
        if elems * esz >= 1 << 63:
            raise PackError(f"safetensors: tensor {name!r}: shape {shape} byte size overflows")
        begin, end = (int(x) for x in entry.get("data_offsets", [0, -1]))
        if begin < 0 or end < begin or end > len(data):
            raise PackError(f"safetensors: tensor {name!r}: offsets [{begin},{end}) outside data "
                            f"section of {len(data)} bytes")
        if end - begin != elems * esz:
            raise PackError(f"safetensors: tensor {name!r}: shape {shape} × {dtype} needs "
                            f"{elems * esz} bytes, offsets span {end - begin}")
        arr = np.frombuffer(data[begin:end], dtype=npdt).reshape(shape)
        if dtype == "F16" and not keep_f16:
            arr = arr.astype(np.float32)
        tensors[name] = arr
        spans.append((begin, end, name))
    cursor = 0
    for begin, end, name in sorted(spans):
        if begin != cursor:
            raise PackError(f"safetensors: tensor {name!r} begins at {begin}, expected {cursor} "
                            "(overlap or gap)")
        cursor = end
    if cursor != len(data):
        raise PackError(f"safetensors: data section is {len(data)} bytes but tensors cover {cursor}")
    return tensors


@dataclasses.dataclass
class Pack:
    cfg: PackConfig
    tensors: Dict[str, np.ndarray]
    manifest: dict


def load_pack(pack_dir: os.PathLike, keep_f16: bool = True) -> Pack:
    """LoadModel's host half (model.go:112-132): manifest, config, tensors."""
    man = load_and_verify_manifest(pack_dir)
    cfg = load_pack_config(pack_dir)
    if man.get("model_id") != cfg.model_id:
        raise PackError(f"pack {cfg.model_id}: manifest is for {man.get('model_id')!r} — mixed "
                        "pack contents")
    raw = (Path(pack_dir) / "model.safetensors").read_bytes()
    try:
        tensors = parse_safetensors(raw, keep_f16=keep_f16)
    except PackError as e:
        raise PackError(f"pack {cfg.model_id}: {e}") from e
    verify_tensor_names(man, tensors)
    return Pack(cfg=cfg, tensors=tensors, manifest=man)


def expected_tensor_shapes(cfg: PackConfig) -> Dict[str, tuple]:
    """Canonical names and shapes newModel requires (model.go:189-257);
    optional biases are included (the caller drops those a pack omits)."""
    h, inter = cfg.hidden_size, cfg.intermediate_size
    out = {"embeddings.word": (cfg.vocab_size, h)}
    if cfg.position_encoding == POS_ABSOLUTE:
        out["embeddings.position"] = (cfg.max_seq_len, h)
    if cfg.type_vocab_size > 0:
        out["embeddings.token_type"] = (cfg.type_vocab_size, h)
    out["embeddings.norm.weight"] = (h,)
    out["embeddings.norm.bias"] = (h,)
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        out[p + "attn.qkv.weight"] = (3 * h, h)
        out[p + "attn.qkv.bias"] = (3 * h,)
        out[p + "attn.out.weight"] = (h, h)
        out[p + "attn.out.bias"] = (h,)
        out[p + "norm1.weight"] = (h,)
        out[p + "norm1.bias"] = (h,)
        out[p + "mlp.fc1.weight"] = (inter, h)
        out[p + "mlp.fc1.bias"] = (inter,)
        if cfg.activation == ACT_SWIGLU:
            out[p + "mlp.gate.weight"] = (inter, h)
            out[p + "mlp.gate.bias"] = (inter,)
        out[p + "mlp.fc2.weight"] = (h, inter)
        out[p + "mlp.fc2.bias"] = (h,)
        out[p + "norm2.weight"] = (h,)
        out[p + "norm2.bias"] = (h,)
    return out


def safetensors_bytes(tensors: Dict[str, np.ndarray]) -> bytes:
    """Serialises tensors (F32/F16) in name order, offsets tiling the data."""
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        arr = np.ascontiguousarray(tensors[name])
        if arr.dtype == np.float32:
            dt = "F32"
        elif arr.dtype == np.float16:
            dt = "F16"
        else:
            raise PackError(f"tensor {name!r}: dtype {arr.dtype} not writable")
        b = arr.astype(arr.dtype.newbyteorder("<"), copy=False).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    return struct.pack("<Q", len(hj)) + hj + b"".join(blobs)


def write_pack(pack_dir: os.PathLike, cfg: PackConfig, tensors: Dict[str, np.ndarray],
               vocab: List[str], created_by: str = "futon_b200.pack") -> Path:
    """Writes a complete, manifest-verified pack."""
    d = Path(pack_dir)
    d.mkdir(parents=True, exist_ok=True)
    (d / "config.json").write_text(json.dumps(cfg.to_dict(), indent=2, sort_keys=True) + "\n")
    (d / "model.safetensors").write_bytes(safetensors_bytes(tensors))
    (d / "vocab.txt").write_text("\n".join(vocab) + "\n")
    members = {m: {"sha256": sha256_file(d / m), "size": (d / m).stat().st_size}
               for m in MANIFEST_MEMBERS}
    man = {"created_by": created_by, "members": members, "model_id": cfg.model_id,
           "pack_format": cfg.pack_format, "tensor_names": sorted(tensors)}
    (d / "manifest.json").write_text(json.dumps(man, indent=2, sort_keys=True) + "\n")
    return d

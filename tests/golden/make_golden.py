"""Regenerates tests/golden/ from the reference checkout.

Copies the reference's toy weight packs (native/testdata/toy/<pack>/:
config.json, model.safetensors, manifest.json, vocab.txt) and their golden
vectors (native/testdata/toy/expected.json, produced upstream by
scripts/gen-native-embed-fixtures.py from transformers BertModel and the
pinned nomic-bert code) byte for byte, so the parity tests run where the
reference tree is absent. Also records the oracle's vectors for the same
cases (oracle_vectors.json) as a regression pin.

Also copies the tokenizer conformance fixtures (native/testdata/
tokenizer_fixtures.json: ids the HF fast BERT tokenizer produced for the
reference's fixture texts, at each pack's max length and at 16) and the
bert-base-uncased vocab they were made with (native/testdata/
vocab_bert_uncased.txt) into tokenizer/, refusing a vocab whose sha256
differs from the value the reference's tests record for it
(native/tokenizer_test.go:18).

Usage: python tests/golden/make_golden.py /path/to/futon-checkout
"""
from __future__ import annotations

import hashlib
import json
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
PACKS = ("toy-absolute-gelu", "toy-rope-swiglu")
MEMBERS = ("config.json", "model.safetensors", "manifest.json", "vocab.txt")
TOKENIZER_FILES = ("tokenizer_fixtures.json", "vocab_bert_uncased.txt")
VOCAB_SHA256 = "07eced375cec144d27c900241f3e339478dec958f92fddbc551f295c992038a3"


def copy_tokenizer_fixtures(ref: Path) -> None:
    src = ref / "native" / "testdata"
    dst = HERE / "tokenizer"
    dst.mkdir(parents=True, exist_ok=True)
    got = hashlib.sha256((src / "vocab_bert_uncased.txt").read_bytes()).hexdigest()
    if got != VOCAB_SHA256:
        raise SystemExit(f"vocab_bert_uncased.txt sha256 {got} != recorded {VOCAB_SHA256}")
    for f in TOKENIZER_FILES:
        shutil.copyfile(src / f, dst / f)
    digest = {f: hashlib.sha256((dst / f).read_bytes()).hexdigest() for f in TOKENIZER_FILES}
    (dst / "SHA256SUMS.json").write_text(json.dumps(digest, indent=1, sort_keys=True) + "\n")


def main(ref: Path) -> None:
    src = ref / "native" / "testdata" / "toy"
    dst = HERE / "toy"
    dst.mkdir(parents=True, exist_ok=True)
    for pack in PACKS:
        (dst / pack).mkdir(exist_ok=True)
        for m in MEMBERS:
            shutil.copyfile(src / pack / m, dst / pack / m)
    shutil.copyfile(src / "expected.json", dst / "expected.json")

    sys.path.insert(0, str(ROOT))
    from futon_b200.pack import load_pack
    from oracle.oracle import OracleModel

    exp = json.loads((dst / "expected.json").read_text())
    out = {}
    for pack, pexp in exp["packs"].items():
        p = load_pack(dst / pack, keep_f16=False)
        m = OracleModel(p.cfg, p.tensors)
        rec = {"forward_cases": [], "matryoshka_cases": []}
        for c in pexp["forward_cases"]:
            rec["forward_cases"].append({"ids": c["ids"], "vector": m.encode(c["ids"]).tolist()})
        for c in pexp.get("matryoshka_cases", []):
            rec["matryoshka_cases"].append(
                {"ids": c["ids"], "dim": c["dim"], "vector": m.encode(c["ids"], c["dim"]).tolist()})
        out[pack] = rec
    (dst / "oracle_vectors.json").write_text(json.dumps(out, indent=1) + "\n")
    digest = {f.relative_to(dst).as_posix(): hashlib.sha256(f.read_bytes()).hexdigest()
              for f in sorted(dst.rglob("*")) if f.is_file() and f.name != "SHA256SUMS.json"}
    (dst / "SHA256SUMS.json").write_text(json.dumps(digest, indent=1, sort_keys=True) + "\n")
    copy_tokenizer_fixtures(ref)
    print(f"wrote {dst} and {HERE / 'tokenizer'}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/futon-checkout")
    main(Path(sys.argv[1]))

"""Text in, vectors out: the Provider's Embed / EmbedBatch over the native
tokenizer and the CUDA forward (native/model_test.go: TestToyProviderEndToEnd,
TestBatchMatchesSingle; native/provider.go:69-121, 152-202)."""
from __future__ import annotations

import random

import numpy as np
import pytest

from conftest import GOLDEN, GPU_COSINE_MIN, cosine
from futon_b200 import FutonError, Options, Provider, provider as P
from futon_b200.pack import load_pack, write_pack
from oracle import tokenizer as OT

pytestmark = pytest.mark.gpu


def test_toy_provider_end_to_end(gpu, toy_expected):
    """Text → tokenizer → forward against the upstream vectors (HF tokenizer
    + upstream model), the empty string and an [UNK] text included."""
    p = Provider(Options(pack_dir=str(GOLDEN / "toy-absolute-gelu"), devices=[0]))
    try:
        cases = toy_expected["packs"]["toy-absolute-gelu"]["text_cases"]
        assert len(cases) == 4
        max_len = p.model.effective_max_seq_len()
        for c in cases:
            assert p.tokenizer.encode(c["text"], max_len) == c["ids"], c["text"]
            got = p.embed(c["text"])
            want = np.asarray(c["vector"], np.float32)
            assert got.shape == want.shape
            assert cosine(got, want) >= GPU_COSINE_MIN, (c["text"], cosine(got, want))
    finally:
        p.close()


def test_text_batch_matches_single(gpu):
    """EmbedBatch is bit-identical to Embed per text (TestBatchMatchesSingle)."""
    p = Provider(Options(pack_dir=str(GOLDEN / "toy-rope-swiglu"), devices=[0]))
    try:
        texts = ["the cat sat on the mat.", "hello", "", "snowman runs",
                 "the the the the the the the the", "unaffable!"]
        batch = p.embed_batch(texts)
        assert batch.shape == (len(texts), p.dimensions())
        for i, t in enumerate(texts):
            single = p.embed(t)
            assert np.array_equal(single.view(np.uint32), batch[i].view(np.uint32)), t
    finally:
        p.close()


def test_pipelined_batch_matches_whole_batch(gpu, monkeypatch):
    """A batch cut into chunks (tokenised while the previous chunk encodes)
    gives the vectors of one whole-batch call, and those of the ids path on
    the oracle tokenizer's ids."""
    pack = GOLDEN / "toy-absolute-gelu"
    p = Provider(Options(pack_dir=str(pack), devices=[0]))
    try:
        words = [w for w in (pack / "vocab.txt").read_text().split("\n")
                 if w.isalpha()] + ["?", "Hello", "\u2603", "x" * 120]
        rng = random.Random(5)
        texts = [" ".join(rng.choice(words) for _ in range(rng.randint(0, 70)))
                 for _ in range(600)]
        whole = p.embed_batch(texts)
        monkeypatch.setattr(P, "FIRST_CHUNK_BYTES", 2000)
        assert len(P.text_chunks(texts, P.FIRST_CHUNK_BYTES)) >= 4
        chunked = p.embed_batch(texts)
        assert np.array_equal(whole.view(np.uint32), chunked.view(np.uint32))
        cfg = p.model.cfg
        ot = OT.Tokenizer((pack / "vocab.txt").read_bytes(),
                          OT.TokenizerConfig.from_dict(cfg.tokenizer))
        seqs = [ot.encode(t, cfg.effective_max_seq_len()) for t in texts]
        by_ids = p.embed_batch_ids(seqs)
        assert np.array_equal(whole.view(np.uint32), by_ids.view(np.uint32))
    finally:
        p.close()


def test_provider_rejects_vocab_larger_than_pack(gpu, tmp_path):
    """New: vocab.txt with more entries than the pack's vocab_size fails
    (provider.go:83-85)."""
    src = load_pack(GOLDEN / "toy-absolute-gelu", keep_f16=False)
    vocab = (GOLDEN / "toy-absolute-gelu" / "vocab.txt").read_text().split("\n")
    vocab = [v for v in vocab if v] + [f"extra{i}" for i in range(src.cfg.vocab_size)]
    write_pack(tmp_path / "pack", src.cfg, src.tensors, vocab)
    with pytest.raises(FutonError, match="vocab.txt has .* entries but pack declares"):
        Provider(Options(pack_dir=str(tmp_path / "pack"), devices=[0]))

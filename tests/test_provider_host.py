"""Host-side lifecycle of futon_b200.Model, with the native calls replaced by
fakes (no GPU): close() waits for calls in flight on other threads before it
releases the native model, and refuses calls after it (the reference's
Provider.Close lets in-flight forwards finish, native/provider.go:274-281)."""
from __future__ import annotations

import ctypes as C
import threading
import time
import types

import numpy as np
import pytest

from conftest import ROOT
from futon_b200 import FutonError, Model, _lib


class FakeNative:
    def __init__(self, encode_seconds: float):
        self.encode_seconds = encode_seconds
        self.events = []
        self.entered = threading.Event()

    def call(self, name, *args):
        if name == "futon_cuda_encode":
            self.events.append(("encode-start", time.monotonic()))
            self.entered.set()
            time.sleep(self.encode_seconds)
            self.events.append(("encode-end", time.monotonic()))
        return 0

    def lib(self):
        fake = self

        class L:
            @staticmethod
            def futon_cuda_model_destroy(h):
                fake.events.append(("destroy", time.monotonic()))

        return L


@pytest.fixture
def fake_model(monkeypatch):
    native = FakeNative(encode_seconds=0.3)
    monkeypatch.setattr(_lib, "call", native.call)
    monkeypatch.setattr(_lib, "lib", native.lib)
    m = Model.__new__(Model)
    m.cfg = types.SimpleNamespace(hidden_size=8)
    m._init_handle(C.c_void_p(0x1000))
    return m, native


def test_close_waits_for_inflight_call(fake_model):
    m, native = fake_model
    ids, cu = np.array([101, 5, 102], np.int32), np.array([0, 3], np.int32)
    t = threading.Thread(target=m.encode_packed, args=(ids, cu))
    t.start()
    assert native.entered.wait(5)
    m.close()  # must block until the encode returns
    t.join(5)
    kinds = [k for k, _ in native.events]
    assert kinds == ["encode-start", "encode-end", "destroy"], kinds
    with pytest.raises(FutonError, match="model is closed"):
        m.encode_packed(ids, cu)


def test_close_is_idempotent(fake_model):
    m, native = fake_model
    m.close()
    m.close()
    assert [k for k, _ in native.events] == ["destroy"]


# ---- text path: chunked, pipelined tokenisation (host logic only) ----------

def test_text_chunks_cover_batch_and_double():
    from futon_b200.provider import text_chunks
    texts = ["x" * 100] * 1000  # 100,000 bytes
    ch = text_chunks(texts, first_bytes=5000)
    assert ch[0][0] == 0 and ch[-1][1] == len(texts)
    assert all(a[1] == b[0] for a, b in zip(ch, ch[1:]))
    sizes = [hi - lo for lo, hi in ch]
    # 50, 100, 200 texts; the 65,000 bytes left are under twice the next
    # chunk's 40,000, so the last chunk takes them all.
    assert sizes == [50, 100, 200, 650]
    assert text_chunks(texts, first_bytes=60000) == [(0, 1000)]
    assert text_chunks([], first_bytes=10) == []
    assert text_chunks(["y" * 50], first_bytes=10) == [(0, 1)]


class _IdsModel:
    """Stands in for Model: each vector is a function of its sequence's ids."""

    def __init__(self):
        self.calls = []

    def effective_max_seq_len(self):
        return 32

    def out_width(self, out_dim):
        return out_dim or 4

    def encode_batch(self, ids, cu, out_dim=0, cancel=None, out=None):
        self.calls.append(len(cu) - 1)
        for i in range(len(cu) - 1):
            s = ids[cu[i]:cu[i + 1]].astype(np.float64)
            out[i] = 0
            out[i, :4] = [len(s), s.sum(), (s * np.arange(1, len(s) + 1)).sum(), s[-2]]
        return out


def test_embed_texts_chunked_equals_whole(monkeypatch):
    import random
    from futon_b200 import provider as P
    from futon_b200.tokenizer import Tokenizer, TokenizerConfig
    vocab = (ROOT / "tests" / "golden" / "tokenizer" / "vocab_bert_uncased.txt").read_bytes()
    tok = Tokenizer(vocab, TokenizerConfig(do_lower_case=True, tokenize_chinese_chars=True))
    rng = random.Random(3)
    words = ["the", "cat", "Sat", "on", "unaffable", "mat.", "été", "自然", ""]
    texts = [" ".join(rng.choice(words) for _ in range(rng.randint(0, 40))) for _ in range(500)]
    whole_model = _IdsModel()
    whole = P.embed_texts(whole_model, tok, texts)
    assert whole_model.calls == [500]
    monkeypatch.setattr(P, "FIRST_CHUNK_BYTES", 1500)
    chunked_model = _IdsModel()
    chunked = P.embed_texts(chunked_model, tok, texts, threads=2)
    assert len(chunked_model.calls) >= 3 and sum(chunked_model.calls) == 500
    assert np.array_equal(whole, chunked)
    seqs = [tok.encode(t, 32) for t in texts]
    assert [int(v) for v in whole[:, 0]] == [len(s) for s in seqs]
    assert P.embed_texts(_IdsModel(), tok, []).shape == (0, 4)


# ---- Provider text API over a stand-in model (host logic only) -------------

class _FakePackModel(_IdsModel):
    """Model.load's stand-in: the pack's config, vectors from _IdsModel."""

    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        self.closed = False

    def effective_max_seq_len(self):
        return self.cfg.effective_max_seq_len()

    def encode_tokens(self, ids, out_dim=0, device=0, cancel=None):
        ids = np.asarray(ids, np.int32)
        out = np.empty((1, self.out_width(out_dim)), np.float32)
        return self.encode_batch(ids, np.array([0, ids.size], np.int32), out_dim, cancel, out)[0]

    def close(self):
        self.closed = True


def _provider(monkeypatch, pack_dir):
    from futon_b200 import provider as P
    from futon_b200.pack import load_pack_config
    made = []

    def load(d, devices=None, q8=None):
        made.append(_FakePackModel(load_pack_config(d)))
        return made[-1]

    monkeypatch.setattr(P.Model, "load", staticmethod(load))
    return P, made


def test_provider_text_api(monkeypatch, toy_expected):
    """Embed / EmbedBatch tokenise with the pack's own vocab and config (the
    toy packs' upstream ids) and give the same rows; calls after Close fail."""
    P, made = _provider(monkeypatch, None)
    pack = ROOT / "tests" / "golden" / "toy" / "toy-absolute-gelu"
    prov = P.Provider(P.Options(pack_dir=str(pack)))
    cases = toy_expected["packs"]["toy-absolute-gelu"]["text_cases"]
    texts = [c["text"] for c in cases]
    batch = prov.embed_batch(texts)
    for i, c in enumerate(cases):
        assert prov.tokenizer.encode(c["text"], 64) == c["ids"]
        single = prov.embed(c["text"])
        assert np.array_equal(single, batch[i])
        ids = np.asarray(c["ids"], np.float64)
        assert single[0] == len(ids) and single[1] == ids.sum()
    assert prov.embed_batch([]).shape == (0, prov.dimensions())
    prov.close()
    assert made[0].closed
    with pytest.raises(FutonError, match="provider is closed"):
        prov.embed("hello")


def test_provider_new_checks_the_vocab(monkeypatch, tmp_path):
    """New (provider.go:69-104): a vocab.txt larger than the pack's
    vocab_size, or none at all, fails and releases the loaded model."""
    from futon_b200.pack import load_pack, write_pack
    P, made = _provider(monkeypatch, None)
    src = load_pack(ROOT / "tests" / "golden" / "toy" / "toy-absolute-gelu", keep_f16=False)
    vocab = [v for v in (ROOT / "tests" / "golden" / "toy" / "toy-absolute-gelu" /
                         "vocab.txt").read_text().split("\n") if v]
    big = write_pack(tmp_path / "big", src.cfg, src.tensors,
                     vocab + [f"extra{i}" for i in range(src.cfg.vocab_size)])
    with pytest.raises(FutonError, match="vocab.txt has .* entries but pack declares vocab_size"):
        P.Provider(P.Options(pack_dir=str(big)))
    assert made[-1].closed
    ok = write_pack(tmp_path / "ok", src.cfg, src.tensors, vocab)
    (ok / "vocab.txt").unlink()
    with pytest.raises(FutonError, match="tokenizer: open vocab"):
        P.Provider(P.Options(pack_dir=str(ok)))
    assert made[-1].closed

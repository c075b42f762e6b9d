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
            out[i] = [len(s), s.sum(), (s * np.arange(1, len(s) + 1)).sum(), s[-2]]
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

"""Host-side parts of bench.py that the driver's GPU run depends on, checked
on the CPU with a stand-in for the model (no GPU needed)."""
from __future__ import annotations

import numpy as np

import bench
from futon_b200 import synth


class _UnitModel:
    """Stands in for Model: unit vectors, one per sequence."""

    def effective_max_seq_len(self):
        return 512

    def out_width(self, out_dim):
        return out_dim or 384

    def encode_batch(self, ids, cu, out_dim=0, cancel=None, out=None):
        assert ids.dtype == np.int32 and cu.dtype == np.int32 and out is not None
        assert ids.size == int(cu[-1]) and len(out) == len(cu) - 1
        out[:] = 0
        out[:, 0] = 1
        return out


def test_text_path_line():
    """The text_path key: tokenizer throughput, text → vectors and the
    tokenizer's CPU baseline (the compiled port, whose ids must equal the
    library's), on synthetic texts that tokenise to exactly their c4
    lengths."""
    r = bench.text_path(_UnitModel(), synth, nseq=1500, steps=1, warmup=0)
    assert set(r) == {"config", "tokenizer", "e2e", "cpu_baseline"}
    assert r["config"].startswith("1500 synthetic texts")
    tk = r["tokenizer"]
    assert tk["texts_per_sec"] > 0 and tk["tokens_per_sec"] > tk["texts_per_sec"]
    assert tk["single_thread_texts_per_sec"] > 0 and tk["threads"] >= 1
    assert r["e2e"]["value"] > 0 and r["e2e"]["unit"] == bench.UNIT
    cb = r["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] == tk["threads"] and cb["value"] > 0
    assert cb["single_thread_texts_per_sec"] > 0


def test_make_texts_tokenise_to_their_lengths():
    from futon_b200.tokenizer import Tokenizer, TokenizerConfig
    vocab = bench.VOCAB_PATH.read_bytes()
    texts, lens = synth.make_texts("c4", vocab.decode().split("\n"), seed=3, nseq=400)
    tok = Tokenizer(vocab, TokenizerConfig(**synth.TOKENIZER))
    ids, cu = tok.encode_batch(texts, 512)
    assert np.array_equal(np.diff(cu), lens)
    want_ids, want_cu = synth.make_inputs("c4", seed=3, nseq=400)
    assert np.array_equal(np.diff(want_cu), lens)  # the same c4 length draw

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

"""Host side of the device status word: a raised timeout bit becomes a
RuntimeError at the next check, and the routers check before each update.
Runs on CPU with a fake library (no GPU, no fault)."""
import contextlib
import ctypes

import pytest
import torch


class _FakeLib:
    def __init__(self, word):
        self.word = word
        self.reads = 0

    def sl_device_status(self, reset, out):
        self.reads += 1
        ctypes.cast(out, ctypes.POINTER(ctypes.c_uint))[0] = self.word
        if reset:
            self.word = 0
        return 0

    def sl_last_error(self):
        return b""


@pytest.fixture
def fake(monkeypatch):
    from sparsecore_b200 import _native as N

    lib = _FakeLib(0)
    monkeypatch.setattr(N, "lib", lambda: lib)
    monkeypatch.setattr(N, "require_cuda", lambda device=None: torch.device("cuda", 0))
    monkeypatch.setattr(torch.cuda, "synchronize", lambda device=None: None)
    monkeypatch.setattr(torch.cuda, "device", lambda d: contextlib.nullcontext())
    return lib


def test_timeout_bit_raises_once_and_clears(fake):
    from sparsecore_b200 import _native as N

    N.check_device_status()  # clean word: no error
    fake.word = 1
    with pytest.raises(RuntimeError, match="timed out"):
        N.check_device_status()
    N.check_device_status()  # the read cleared it
    assert fake.reads == 3


def test_router_checks_status_before_update(fake, monkeypatch):
    from sparsecore_b200 import router as R

    class _Csr:
        values = torch.zeros(1)

    class _Layer:
        _csr = _Csr()

    algo = R.SET(0.9, drop_fraction=0.3, update_freq=2, seed=0)
    algo.layers.append(_Layer())
    updates = []
    monkeypatch.setattr(algo, "update", lambda: updates.append(algo._step_idx))
    algo.step()
    assert fake.reads == 0 and updates == []  # no update, no check
    fake.word = 1
    with pytest.raises(RuntimeError, match="timed out"):
        algo.step()
    assert updates == []  # the update did not run on incomplete gradients

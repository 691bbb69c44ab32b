"""Host logic of the device-fault reporting (spark_gpt_b200/faults.py) on CPU.

The pinned landing slot is replaced by a CPU tensor and the synchronous
clear by a stand-in, so the check that every layer call makes first can be
driven without a GPU: a zero word passes, a non-zero word raises DeviceFault
once, naming each recorded bit, and clears the slot."""

import pytest
import torch

from spark_gpt_b200 import faults


class _FakeWatch:
    def __init__(self):
        self.device = torch.device("cuda", 0)
        self.host = torch.zeros(1, dtype=torch.int32)


@pytest.fixture
def watch(monkeypatch):
    w = _FakeWatch()
    cleared = []

    def clear(wt):
        cleared.append(int(wt.host[0]))
        wt.host.zero_()
        return 0

    monkeypatch.setattr(faults, "_watch", lambda device: w)
    monkeypatch.setattr(faults, "_clear", clear)
    w.cleared = cleared
    return w


def test_no_fault_passes(watch):
    faults.raise_pending("cuda:0")
    assert watch.cleared == []


@pytest.mark.parametrize("word,needles", [
    (1, ["0x1", "bounded device wait gave up"]),
    (2, ["0x2", "expert id outside"]),
    (5, ["0x5", "bounded device wait", "inconsistent sizes"]),
])
def test_a_landed_fault_raises_once_and_clears(watch, word, needles):
    watch.host[0] = word
    with pytest.raises(faults.DeviceFault) as ei:
        faults.raise_pending("cuda:0")
    assert isinstance(ei.value, RuntimeError)
    assert ei.value.word == word
    for n in needles:
        assert n in str(ei.value)
    assert watch.cleared == [word] and int(watch.host[0]) == 0
    faults.raise_pending("cuda:0")  # raised once: the next call passes


def test_public_api():
    import spark_gpt_b200 as pkg
    assert pkg.DeviceFault is faults.DeviceFault and pkg.check_faults is faults.check_faults

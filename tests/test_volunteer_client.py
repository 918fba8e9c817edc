"""Volunteer client (launch/client.py) on CPU with a faked CUDA device: the device is
auto-detected, memory levers are switched on in order until the path fits the free
memory, a path that fits nowhere falls back to the CPU (or refuses a forced device), a
failed memory probe falls back too, and the health line reports throughput.

Behaviour of the reference's ``src/opendipaco/launch/client.py`` (``resolve_device``,
``HealthReporter``)."""

import pytest
import torch

from opendipaco_b200.launch import client as C
from opendipaco_b200.train.memory import vram_breakdown

from helpers import tiny_config


def _fake_cuda(monkeypatch, free_bytes):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    if isinstance(free_bytes, Exception):
        def probe():
            raise free_bytes
    else:
        def probe():
            return free_bytes, 2 * free_bytes
    monkeypatch.setattr(torch.cuda, "mem_get_info", probe)


def test_cpu_without_accelerators():
    d, over, notes = C.resolve_device(tiny_config(), batch_size=4, seq_len=16)
    assert d in ("cpu", "mps") and over == {}
    with pytest.raises(SystemExit):
        C.choose_device(tiny_config(), requested="tpu", batch_size=4, seq_len=16)


def test_levers_switch_on_until_the_path_fits(monkeypatch):
    cfg = tiny_config(hidden=64, vocab=4096, seq=64)
    plain = vram_breakdown(cfg, batch_size=8, seq_len=64)["total"]
    _fake_cuda(monkeypatch, int(10 * plain / C._USABLE_FRACTION))
    roomy = C.choose_device(cfg, batch_size=8, seq_len=64)
    assert roomy.device == "cuda" and roomy.overrides == {}
    smallest = vram_breakdown(cfg, batch_size=8, seq_len=64, autocast=True, checkpoint=True,
                              chunked_logits=True)["total"]
    _fake_cuda(monkeypatch, int((smallest + plain) / 2 / C._USABLE_FRACTION))
    tight = C.choose_device(cfg, batch_size=8, seq_len=64)
    assert tight.device == "cuda" and tight.overrides and any("VRAM fit" in n for n in tight.notes)


def test_too_small_or_unprobeable_devices(monkeypatch):
    cfg = tiny_config()
    _fake_cuda(monkeypatch, 1024)
    assert C.choose_device(cfg, batch_size=4, seq_len=16).device == "cpu"
    with pytest.raises(SystemExit):
        C.choose_device(cfg, requested="cuda", batch_size=4, seq_len=16)
    _fake_cuda(monkeypatch, RuntimeError("driver gone"))
    assert C.choose_device(cfg, batch_size=4, seq_len=16).device == "cpu"


def test_health_line_reports_throughput():
    class _Bucket:
        sent_bytes, recv_bytes = 3_000_000, 1_000_000

    h = C.HealthReporter(target="127.0.0.1:1", device="cuda", bucket=_Bucket(), cap_mbps=20)
    line = h._line(0.0, 10.0, 2.0, 1_000_000)
    assert "4.00/20 Mbps" in line and "4.0 MB total" in line and "up 10s" in line

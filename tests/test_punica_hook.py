"""The reference-API vLLM hook (lora_warp_pipe/punica_wrapper.py:119-159,
219-238 of the reference) over libwp_b200.so.

CPU: the AS_WARP_PIPE opt-in gate and the install rules of
install_warp_pipe_add_lora (no-op without the gate, without a manager or a
wrapper, and when already installed; otherwise the live wrapper's __class__
is reassigned and its state kept).

GPU: a stub lora_manager whose PunicaWrapper is swapped in place; then
update_metadata (the step's segment table) and add_lora, whole-width and
sliced (y_offset / y_slice_size), against the oracle restatement of the
reference's apply math (tests/correctness/test_add_lora_packed.py:35-45).
"""

from __future__ import annotations

import pytest
import torch

from adapterslotsplusplus_b200 import punica_wrapper as pw


class _StubWrapper(pw.FusedPunicaWrapper):
    """Stands in for vLLM's PunicaWrapper instance (the attributes the hook reads)."""

    def __init__(self):
        self.is_prefill = False
        self.token_lora_indices = None
        self.kept = "state"


class _AdapterManager:
    def __init__(self, wrapper):
        self.punica_wrapper = wrapper


class _LoraManager:
    def __init__(self, wrapper):
        self._adapter_manager = _AdapterManager(wrapper)


def test_gate_off_is_noop(monkeypatch):
    monkeypatch.delenv("AS_WARP_PIPE", raising=False)
    w = _StubWrapper()
    assert not pw.warp_pipe_available()
    assert pw.install_warp_pipe_add_lora(_LoraManager(w)) is False
    assert type(w) is _StubWrapper
    monkeypatch.setenv("AS_WARP_PIPE", "0")
    assert pw.install_warp_pipe_add_lora(_LoraManager(w)) is False
    assert type(w) is _StubWrapper


def test_gate_on_installs_once(monkeypatch):
    monkeypatch.setenv("AS_WARP_PIPE", "1")
    assert pw.warp_pipe_available()
    assert pw.install_warp_pipe_add_lora(None) is False

    class NoAdapters:
        _adapter_manager = None

    assert pw.install_warp_pipe_add_lora(NoAdapters()) is False
    assert pw.install_warp_pipe_add_lora(_LoraManager(None)) is False
    w = _StubWrapper()
    mgr = _LoraManager(w)
    assert pw.install_warp_pipe_add_lora(mgr) is True
    assert isinstance(w, pw.FusedPunicaWrapperWarpPipe)
    assert w.kept == "state"  # same instance, class swapped
    assert pw.install_warp_pipe_add_lora(mgr) is False  # already installed


def test_hook_engine_uses_serving_contract(monkeypatch):
    """The hook's engine runs with prefetch_weights, the configuration the
    benchmark reports (checked without creating the engine)."""
    seen = {}

    class FakeEngine:
        def __init__(self, config=None, device=None):
            seen["cfg"] = config

    monkeypatch.setattr(pw, "WarpPipeEngine", FakeEngine)
    monkeypatch.setattr(pw, "_engine", None)
    pw._get_engine()
    assert seen["cfg"].prefetch_weights is True


@pytest.mark.gpu
@pytest.mark.parametrize("rank", [16, 32, 64])
def test_hook_update_metadata_and_add_lora(cuda, monkeypatch, rank):
    from oracle.apply import add_lora_grouped, tolerance

    monkeypatch.setenv("AS_WARP_PIPE", "1")
    monkeypatch.setattr(pw, "_engine", None)
    w = _StubWrapper()
    assert pw.install_warp_pipe_add_lora(_LoraManager(w))
    g = torch.Generator().manual_seed(rank)
    L, d, o, T = 6, 1024, 768, 80
    idx = torch.tensor([0] * 7 + [-1] * 3 + [2] * 40 + [5] * 9 + [1] * 21, dtype=torch.int64)
    assert idx.numel() == T
    dt = torch.bfloat16
    wa = (torch.randn(L, 1, rank, d, generator=g) * 0.02).to(dt)
    wb = (torch.randn(L, 1, o, rank, generator=g) * 0.02).to(dt)
    x = (torch.randn(T, d, generator=g) * 0.1).to(dt)
    y = (torch.randn(T, o, generator=g) * 0.1).to(dt)
    ywide = (torch.randn(T, 3 * o, generator=g) * 0.1).to(dt)

    w.token_lora_indices = idx.to(cuda)
    w.update_metadata(None, None, L, 32000, 0)
    yd = y.to(cuda)
    w.add_lora(yd, x.to(cuda), wa.to(cuda), wb.to(cuda), 0.5)
    ywd = ywide.to(cuda)
    w.add_lora(ywd, x.to(cuda), wa.to(cuda), wb.to(cuda), 0.5, y_offset=o, y_slice_size=o)
    torch.cuda.synchronize()

    ref = add_lora_grouped(y, x, wa, wb, 0.5, idx)
    rms = float(ref.pow(2).mean().sqrt())
    assert float((yd.float().cpu() - ref).abs().max()) <= tolerance(dt) * rms
    refw = add_lora_grouped(ywide, x, wa, wb, 0.5, idx, y_offset=o)
    rmsw = float(refw.pow(2).mean().sqrt())
    assert float((ywd.float().cpu() - refw).abs().max()) <= tolerance(dt) * rmsw
    # columns outside the slice are untouched
    assert torch.equal(ywd.cpu()[:, :o], ywide[:, :o]) and torch.equal(ywd.cpu()[:, 2 * o:], ywide[:, 2 * o:])


@pytest.mark.gpu
def test_hook_rejects_unsupported_rank(cuda, monkeypatch):
    monkeypatch.setenv("AS_WARP_PIPE", "1")
    monkeypatch.setattr(pw, "_engine", None)
    w = _StubWrapper()
    assert pw.install_warp_pipe_add_lora(_LoraManager(w))
    w.token_lora_indices = torch.zeros(8, dtype=torch.int64, device=cuda)
    w.update_metadata(None, None, 1, 32000, 0)
    x = torch.zeros(8, 256, dtype=torch.bfloat16, device=cuda)
    y = torch.zeros(8, 256, dtype=torch.bfloat16, device=cuda)
    wa = torch.zeros(1, 1, 12, 256, dtype=torch.bfloat16, device=cuda)
    wb = torch.zeros(1, 1, 256, 12, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError, match="rank 12"):
        w.add_lora(y, x, wa, wb, 1.0)

"""vLLM 0.22 hook (adapterslotsplusplus_b200.vllm_punica): the mapping of
PunicaWrapperGPU.add_lora_linear / add_shrink / add_expand onto the engine,
checked against vLLM's documented semantics (punica_gpu.py docstrings) with
an engine stand-in that computes with the oracle (CPU), and with the real
engine on the GPU."""

import pytest
import torch

from adapterslotsplusplus_b200 import vllm_punica as vp
from oracle import apply as oa
from tests.golden.cases import zipf_ids

T, D, L, R = 48, 256, 6, 16


class OracleEngine:
    """The engine's live-path methods computed by the oracle for fixed indices."""

    def __init__(self, idx):
        self.idx = torch.as_tensor(idx)
        self.calls = []

    def add_lora(self, y, x, wa, wb, scale, y_offset=None, y_slice_size=None):
        self.calls.append("add_lora")
        off = 0 if y_offset is None else y_offset
        y.copy_(oa.add_lora_grouped(y, x, wa, wb, scale, self.idx, y_offset=off).to(y.dtype))
        return True

    def add_lora_packed_nslice(self, y, x, As, Bs, scale, widths):
        self.calls.append("nslice")
        off = 0
        for a, b, w in zip(As, Bs, widths):
            y.copy_(oa.add_lora_grouped(y, x, a, b, scale, self.idx, y_offset=off).to(y.dtype))
            off += w
        return True

    def add_lora_shrink(self, H, x, wa, scale):
        self.calls.append("shrink")
        for a in self.idx.unique().tolist():
            if a >= 0:
                rows = (self.idx == a).nonzero().reshape(-1)
                H[rows] = (x[rows].float() @ wa[a, 0].float().T) * scale
        return True

    def add_lora_expand(self, y, H, wb, y_offset=0):
        self.calls.append("expand")
        o = wb.size(-2)
        for a in self.idx.unique().tolist():
            if a >= 0:
                rows = (self.idx == a).nonzero().reshape(-1)
                yy = y[rows, y_offset:y_offset + o].float() + H[rows] @ wb[a, 0].float().T
                y[rows, y_offset:y_offset + o] = yy.to(y.dtype)
        return True


def _stacks(widths, dtype=torch.float32, seed=0):
    g = torch.Generator().manual_seed(seed)
    A = [(torch.randn(L, 1, R, D, generator=g) * 0.05).to(dtype) for _ in widths]
    B = [(torch.randn(L, 1, w, R, generator=g) * 0.05).to(dtype) for w in widths]
    x = (torch.randn(T, D, generator=g) * 0.3).to(dtype)
    y = (torch.randn(T, sum(widths), generator=g) * 0.3).to(dtype)
    return A, B, x, y


def _vllm_semantics(y, x, A, B, scale, widths, idx, add_inputs=True):
    """for i: y[:, off_i:off_i+w_i] (+)= (x @ A_i[idx]^T * scale) @ B_i[idx]^T, rows with idx < 0 untouched"""
    out = y.float().clone()
    off = 0
    for a, b, w in zip(A, B, widths):
        for t in range(x.size(0)):
            i = int(idx[t])
            if i < 0:
                if not add_inputs:
                    out[t, off:off + w] = 0
                continue
            v = (x[t].float() @ a[i, 0].float().T) * scale @ b[i, 0].float().T
            out[t, off:off + w] = (out[t, off:off + w] if add_inputs else 0) + v
        off += w
    return out


@pytest.mark.parametrize("widths", [[128, 128], [128, 64, 64], [96]])
@pytest.mark.parametrize("add_inputs", [True, False])
def test_add_lora_linear_mapping(widths, add_inputs):
    idx = zipf_ids(L, T, seed=2)
    idx[5:9] = -1
    A, B, x, y = _stacks(widths)
    eng = OracleEngine(idx)
    want = _vllm_semantics(y, x, A, B, 0.5, widths, idx, add_inputs)
    vp.apply_lora_linear(eng, y, x, A, B, 0.5, widths, add_inputs)
    assert torch.allclose(y, want, atol=1e-5)
    equal = len(set(widths)) == 1 and len(widths) > 1
    assert eng.calls == (["nslice"] if equal else ["add_lora"] * len(widths))


def test_shrink_then_expand_mapping():
    widths = [128, 64]
    idx = zipf_ids(L, T, seed=4)
    idx[0:3] = -1
    A, B, x, y = _stacks(widths, seed=1)
    eng = OracleEngine(idx)
    buf = torch.full((len(widths), T, R), 7.0)  # stale contents: the shrink zeroes it
    vp.apply_shrink(eng, buf, x, A, 0.25)
    assert torch.all(buf[:, 0:3] == 0)
    want = _vllm_semantics(y, x, A, B, 0.25, widths, idx)
    vp.apply_expand(eng, y, buf, B, widths, offset_start=0)
    assert torch.allclose(y, want, atol=1e-5)


def test_slice_lists_must_match():
    A, B, x, y = _stacks([64, 64])
    with pytest.raises(RuntimeError):
        vp.apply_lora_linear(OracleEngine([0] * T), y, x, A, B[:1], 1.0, [64, 64])


def test_install_needs_opt_in(monkeypatch):
    monkeypatch.delenv("AS_WARP_PIPE", raising=False)
    assert vp.install_warp_pipe_punica(object()) is False


@pytest.mark.gpu
@pytest.mark.parametrize("widths", [[1024, 256, 256], [1024, 1024]])
def test_add_lora_linear_on_gpu(cuda, widths):
    """GQA-shaped q/k/v (unequal slices: one launch per slice) and gate/up
    (equal slices: one multi-slice launch) through the real engine."""
    from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine

    d, r, L2, n = 1024, 32, 8, 96
    g = torch.Generator().manual_seed(9)
    A = [(torch.randn(L2, 1, r, d, generator=g) * 0.02).bfloat16() for _ in widths]
    B = [(torch.randn(L2, 1, w, r, generator=g) * 0.02).bfloat16() for w in widths]
    x = (torch.randn(n, d, generator=g) * 0.1).bfloat16()
    y = (torch.randn(n, sum(widths), generator=g) * 0.1).bfloat16()
    idx = torch.as_tensor(zipf_ids(L2, n, seed=6), dtype=torch.int64)
    want = _vllm_semantics(y, x, A, B, 1.0, widths, idx)
    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=1024))
    assert eng.build_seg_bounds(idx.cuda())
    yd = y.cuda()
    vp.apply_lora_linear(eng, yd, x.cuda(), [a.cuda() for a in A], [b.cuda() for b in B], 1.0, widths)
    # the shrink/expand halves into vLLM's fp32 buffer
    y2 = y.cuda()
    buf = torch.empty(len(widths), n, r, dtype=torch.float32, device="cuda")
    vp.apply_shrink(eng, buf, x.cuda(), [a.cuda() for a in A], 1.0)
    vp.apply_expand(eng, y2, buf, [b.cuda() for b in B], widths)
    torch.cuda.synchronize()
    rms = float(want.pow(2).mean().sqrt())
    for got in (yd, y2):
        err = float((got.float().cpu() - want).abs().max())
        assert err <= 2e-2 * rms, f"max_abs_err {err:.3e} > {2e-2 * rms:.3e}"


def test_wrapper_class_extends_vllm_punica_gpu():
    """The hook class is vLLM 0.22's PunicaWrapperGPU with the three LoRA
    linear entry points overridden (vLLM imports without a GPU)."""
    cls = vp.wrapper_class()
    if cls is None:
        pytest.skip("vLLM's PunicaWrapperGPU does not import here")
    base = cls.__mro__[1]
    assert base.__name__ == "PunicaWrapperGPU"
    for name in ("update_metadata", "add_lora_linear", "add_shrink", "add_expand"):
        assert getattr(cls, name) is not getattr(base, name)

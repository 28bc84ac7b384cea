"""TEST INFRASTRUCTURE ONLY -- torch fp32 restatement of the apply math.

reference_bgmv_shrink / reference_bgmv_expand restate
tests/correctness/reference_bgmv.py:4-18 of the reference:
    H = (X.float() @ A.float().T) * alpha      (alpha applied once, in shrink)
    Y = Y.float() + H.float() @ B.float().T
reference_add_lora restates tests/correctness/test_add_lora_packed.py:35-45:
per row i with idx[i] >= 0, y[i] += (x[i] @ wa[idx,0].T * scale) @ wb[idx,0].T.

apply_segments runs the same math per segment of a table, as the
reference's per-segment checks do (test_bgmv_correctness.py:38-44), with no
rounding of H -- the parity criterion of this build.
"""

from __future__ import annotations

import torch


def reference_bgmv_shrink(X: torch.Tensor, A: torch.Tensor, alpha_scale: float) -> torch.Tensor:
    return (X.float() @ A.float().T) * alpha_scale


def reference_bgmv_expand(H: torch.Tensor, B: torch.Tensor, Y_base: torch.Tensor) -> torch.Tensor:
    return Y_base.float() + (H.float() @ B.float().T)


def reference_add_lora(y, x, wa_t_all, wb_t_all, scale, indices):
    """Row loop; fine for small T (see add_lora_grouped for large T)."""
    y_ref = y.float().clone()
    for i in range(x.shape[0]):
        idx = int(indices[i])
        if idx < 0:
            continue
        a = wa_t_all[idx].reshape(wa_t_all.shape[-2], wa_t_all.shape[-1]).float()
        b = wb_t_all[idx].reshape(wb_t_all.shape[-2], wb_t_all.shape[-1]).float()
        h = (x[i].float() @ a.T) * scale
        y_ref[i] += h @ b.T
    return y_ref


def add_lora_grouped(y, x, wa_t_all, wb_t_all, scale, indices, y_offset: int = 0):
    """Same result as reference_add_lora, grouped by adapter id (fast on CPU).
    Returns fp32 y with the update in columns [y_offset, y_offset + o)."""
    y_ref = y.float().clone()
    idx = torch.as_tensor(indices).reshape(-1).long()
    xf = x.reshape(-1, x.shape[-1])
    o = wb_t_all.shape[-2]
    for a_id in torch.unique(idx).tolist():
        if a_id < 0:
            continue
        rows = torch.nonzero(idx == a_id).reshape(-1)
        a = wa_t_all[a_id].reshape(wa_t_all.shape[-2], wa_t_all.shape[-1]).float()
        b = wb_t_all[a_id].reshape(wb_t_all.shape[-2], wb_t_all.shape[-1]).float()
        h = (xf[rows].float() @ a.T) * scale
        y_ref[rows, y_offset:y_offset + o] += h @ b.T
    return y_ref


def apply_segments(Y, X, table, A_of, B_of, alpha_of):
    """Registry-path oracle. table: iterable of (adapter_id, start, count);
    A_of/B_of/alpha_of map an adapter id to its A [r,d], B [o,r], alpha.
    Returns (H fp32 [T, r], Y fp32)."""
    T = X.shape[0]
    r = None
    Hs = {}
    Yf = Y.float().clone()
    for aid, s, n in table:
        aid, s, n = int(aid), int(s), int(n)
        if n <= 0:
            continue
        h = reference_bgmv_shrink(X[s:s + n], A_of(aid), alpha_of(aid))
        r = h.shape[1]
        Hs[(s, n)] = h
        Yf[s:s + n] = reference_bgmv_expand(h, B_of(aid), Yf[s:s + n])
    H = torch.zeros(T, r or 1, dtype=torch.float32)
    for (s, n), h in Hs.items():
        H[s:s + n] = h
    return H, Yf


def tolerance(dtype: torch.dtype) -> float:
    """Max-abs error bound as a fraction of RMS(Y): 2e-2 for bf16, 5e-3 for fp16."""
    return 2e-2 if dtype == torch.bfloat16 else 5e-3

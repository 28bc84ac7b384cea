"""Multi-tenant draft step: a small decoder whose LoRA projections run the
grouped apply over an AdapterPool.

The reference's draft-side integration wraps a draft model's linears so that
every tenant's draft-LoRA is applied to the whole batch in one pass per layer
(BGMVLoRALinear / wrap_draft, benchmarks/e2e/serve_multitenant.py:56-120)
and captures the draft step in a CUDA graph (benchmarks/kernel/
bench_graph_capture.py:47-103). Here the base linears are plain GEMMs and
each projection's LoRA is one add_lora call of this library on the pool's
stacked slots; the step's segment table (tokens sorted by tenant) is built
once per step and shared by all 7 x layers calls.

DraftDecoder is random-init (no checkpoint): RMSNorm, multi-head attention
over each sequence's lookahead tokens (causal), SwiGLU MLP, an optional LM
head. `lora="pool"` uses the library, `lora="torch"` a plain-torch per-token
gather of the same adapters (the stock path the grouped apply replaces, for
comparison and tests), `lora="none"` the base model alone.
"""

from __future__ import annotations

import math
from typing import List, Optional

import torch
import torch.nn.functional as F

PROJ_NAMES = ("q", "k", "v", "o", "gate", "up", "down")


class DraftDecoder:
    def __init__(self, layers: int = 12, hidden: int = 768, heads: int = 12, inter: int = 3072, vocab: int = 0,
                 device="cuda", dtype=torch.bfloat16, seed: int = 0):
        self.layers, self.hidden, self.heads, self.inter, self.vocab = layers, hidden, heads, inter, vocab
        self.dtype = dtype
        g = torch.Generator(device=device).manual_seed(seed)

        def w(o, i):
            return (torch.randn(o, i, device=device, generator=g) * (1.0 / math.sqrt(i))).to(dtype)

        self.w = []
        for _ in range(layers):
            self.w.append({"q": w(hidden, hidden), "k": w(hidden, hidden), "v": w(hidden, hidden),
                           "o": w(hidden, hidden), "gate": w(inter, hidden), "up": w(inter, hidden),
                           "down": w(hidden, inter)})
        self.lm_head = w(vocab, hidden) if vocab else None

    def dims(self) -> List[tuple]:
        """(d_in, d_out) of the LoRA projections, in call order (layer-major)."""
        h, i = self.hidden, self.inter
        per = [(h, h), (h, h), (h, h), (h, h), (h, i), (h, i), (i, h)]
        return [p for _ in range(self.layers) for p in per]

    @staticmethod
    def _rms(x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(x.dtype)

    def forward(self, x: torch.Tensor, seq_len: int, lora: str = "none", pool=None, scale: float = 1.0,
                torch_lora: Optional[dict] = None) -> torch.Tensor:
        """x [T, hidden] (T = sequences x seq_len, sequences adapter-sorted).
        lora "pool": pool.add_lora per projection (the segment table must be
        built for this step); "torch": torch_lora = {"ids": [T] adapter ids,
        "A": [p] -> [n_adapters, r, d], "B": [p] -> [n_adapters, o, r]}."""
        T, H = x.shape
        nh, hd = self.heads, H // self.heads

        def proj(p, name, inp, W):
            out = F.linear(inp, W)
            if lora == "pool":
                pool.add_lora(p, out, inp, scale)
            elif lora == "torch":
                ids = torch_lora["ids"]
                valid = (ids >= 0)
                A = torch_lora["A"][p][ids.clamp(min=0)]  # [T, r, d]
                B = torch_lora["B"][p][ids.clamp(min=0)]  # [T, o, r]
                h = torch.einsum("td,trd->tr", inp.float(), A.float()) * scale
                # H enters the expand in the weights' 16-bit type, as the
                # stock bgmv_expand and this library's kernels take it
                h = h.to(inp.dtype).float()
                d = torch.einsum("tr,tor->to", h, B.float()) * valid.unsqueeze(1)
                out = (out.float() + d).to(out.dtype)
            return out

        for li, L in enumerate(self.w):
            base = li * len(PROJ_NAMES)
            h = self._rms(x)
            q = proj(base + 0, "q", h, L["q"])
            k = proj(base + 1, "k", h, L["k"])
            v = proj(base + 2, "v", h, L["v"])
            q = q.view(-1, seq_len, nh, hd).transpose(1, 2)
            k = k.view(-1, seq_len, nh, hd).transpose(1, 2)
            v = v.view(-1, seq_len, nh, hd).transpose(1, 2)
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
            a = a.transpose(1, 2).reshape(T, H).contiguous()
            x = x + proj(base + 3, "o", a, L["o"])
            h2 = self._rms(x)
            g = proj(base + 4, "gate", h2, L["gate"])
            u = proj(base + 5, "up", h2, L["up"])
            m = (F.silu(g.float()) * u.float()).to(x.dtype).contiguous()
            x = x + proj(base + 6, "down", m, L["down"])
        x = self._rms(x)
        if self.lm_head is not None:
            return F.linear(x, self.lm_head)
        return x

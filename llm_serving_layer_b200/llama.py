"""
Random-init Llama-3.2-1B with the engine's ``forward_varlen(tokens, meta,
backend)`` contract — the caller the paged-KV path plugs into.

The reference drives the hot path from ``Scheduler.step`` →
``model.forward_varlen(tokens, meta, backend)`` (``serving/scheduler/
scheduler.py:752-757``); the engine that implements it
(``vendor/llm_inference_engine``, ``LlamaModelGPU``) is not part of the
reference tree and no weights ship with it. This module is a stand-in with the
same structure and interface (``docs/ARCHITECTURE.md:167-172``: per layer
project Q/K/V, RoPE at ``meta.positions``, ``backend.append_kv`` then
``backend.attend``, output projection, residual; logits gathered at
``meta.last_token_ix``; with a backend that takes ``rope=``, the RoPE, append
and attention of a layer are one ``append_attend`` call, one kernel launch for
a decode step), at Llama-3.2-1B geometry: hidden 2048, 16 layers,
32 query / 8 KV heads of 64, SwiGLU FFN 8192, vocab 128256, RMSNorm eps 1e-5,
RoPE theta 500000 (plain rotary frequencies, no long-context rescaling), tied
input/output embedding, fp16. Weights are drawn from a seeded N(0, init_std²).

Two options serve exact greedy comparisons. With i.i.d. Gaussian embedding
rows, the 128256 logits of a random model are nearly flat (top-1/top-2 gaps
of a few 1e-3 are common), so any rounding difference upstream flips ties;
``row_norm_sigma`` scales each embedding row by exp(N(0, sigma²)) — a
heavy-tailed spread of token norms, as trained vocabularies have — which
separates the top logits. ``fp32_head`` computes the logits in fp32 (an fp32
copy of the tied head), so they carry no fp16 rounding ties.

The dense parts (projections, FFN, logits) are plain cuBLAS GEMMs through
torch; only attention and the KV write go through the backend.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class LlamaConfig:
    hidden: int = 2048
    n_layers: int = 16
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 64
    ffn: int = 8192
    vocab: int = 128256
    rope_theta: float = 500000.0
    eps: float = 1e-5
    rope_positions: int = 16384  # rows of the cosine / sine tables (largest position + 1)


class RandomLlama:
    """Llama-3.2-1B-shaped decoder with seeded random weights."""

    def __init__(self, cfg: LlamaConfig = LlamaConfig(), device: str | torch.device = "cuda:0",
                 dtype: torch.dtype = torch.float16, seed: int = 0, init_std: float = 0.02,
                 row_norm_sigma: float = 0.0, fp32_head: bool = False, fused_rope: bool = True):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        g = torch.Generator(device=self.device).manual_seed(seed)
        H, Hq, Hkv, Dh = cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim

        def w(*shape):
            return (torch.randn(*shape, generator=g, device=self.device) * init_std).to(dtype)

        self.embed = w(cfg.vocab, H)                 # tied with the output head
        if row_norm_sigma > 0:
            rn = torch.exp(torch.randn(cfg.vocab, 1, generator=g, device=self.device) * row_norm_sigma)
            self.embed = (self.embed.float() * rn).to(dtype)
        self.head32 = self.embed.float() if fp32_head else None
        self.w_qkv = [w((Hq + 2 * Hkv) * Dh, H) for _ in range(cfg.n_layers)]
        self.w_o = [w(H, Hq * Dh) for _ in range(cfg.n_layers)]
        self.w_gate_up = [w(2 * cfg.ffn, H) for _ in range(cfg.n_layers)]
        self.w_down = [w(H, cfg.ffn) for _ in range(cfg.n_layers)]
        ones = torch.ones(H, device=self.device, dtype=dtype)
        self.ln_attn = [ones.clone() for _ in range(cfg.n_layers)]
        self.ln_ffn = [ones.clone() for _ in range(cfg.n_layers)]
        self.ln_final = ones.clone()
        self.inv_freq = 1.0 / (cfg.rope_theta ** (
            torch.arange(0, Dh, 2, device=self.device, dtype=torch.float32) / Dh))
        # cosine / sine tables [rope_positions, Dh / 2]: the same fp32 products
        # position * inv_freq as the per-step computation below, so the same bits
        ang = torch.arange(cfg.rope_positions, device=self.device, dtype=torch.float32)[:, None] \
            * self.inv_freq[None, :]
        self.rope_cos, self.rope_sin = torch.cos(ang).contiguous(), torch.sin(ang).contiguous()
        # with a backend that takes rope= (B200PagedBackend), q and k go to it
        # unrotated and the rotation runs in its kernels (inside the decode
        # launch for a decode step); otherwise torch rotates them here
        self.fused_rope = fused_rope
        self.scale = Dh ** -0.5

    def param_bytes(self) -> int:
        ts = [self.embed, *self.w_qkv, *self.w_o, *self.w_gate_up, *self.w_down]
        return sum(t.numel() * t.element_size() for t in ts)

    def _norm(self, x: torch.Tensor, wgt: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg.eps)).to(self.dtype) * wgt

    def _rope(self, t: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        half = t.shape[-1] // 2
        a, b = t[..., :half].float(), t[..., half:].float()
        return torch.cat([a * cos - b * sin, a * sin + b * cos], dim=-1).to(self.dtype)

    @torch.no_grad()
    def forward_varlen(self, tokens: torch.Tensor, meta: Any, backend: Any) -> torch.Tensor:
        """tokens: (T,) int token ids of every sequence's new tokens packed in
        sequence order; returns (n_seqs, vocab) logits (fp32) of each
        sequence's last token."""
        cfg = self.cfg
        T = tokens.shape[0]
        Hq, Hkv, Dh = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        fused = self.fused_rope and hasattr(backend, "append_attend") and hasattr(backend, "rope")
        if not fused:
            pos = meta.positions.to(self.device).float()
            ang = pos[:, None] * self.inv_freq[None, :]
            cos, sin = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
        x = self.embed[tokens.to(self.device).long()]
        for layer in range(cfg.n_layers):
            h = self._norm(x, self.ln_attn[layer])
            qkv = F.linear(h, self.w_qkv[layer])
            v = qkv[:, (Hq + Hkv) * Dh:].reshape(T, Hkv, Dh)
            if fused:  # RoPE, KV-append and attention in the backend (one launch for a decode step)
                q = qkv[:, : Hq * Dh].reshape(T, Hq, Dh)
                k = qkv[:, Hq * Dh: (Hq + Hkv) * Dh].reshape(T, Hkv, Dh)
                o = backend.append_attend(layer, k, v, q, self.scale, meta, rope=(self.rope_cos, self.rope_sin))
            else:
                q = self._rope(qkv[:, : Hq * Dh].view(T, Hq, Dh), cos, sin)
                k = self._rope(qkv[:, Hq * Dh: (Hq + Hkv) * Dh].view(T, Hkv, Dh), cos, sin)
                if hasattr(backend, "append_attend"):  # one call (one launch for a decode step)
                    o = backend.append_attend(layer, k, v, q, self.scale, meta)
                else:
                    backend.append_kv(layer, k, v, meta)
                    o = backend.attend(q, layer, self.scale, meta)
            x = x + F.linear(o.reshape(T, Hq * Dh), self.w_o[layer])
            h = self._norm(x, self.ln_ffn[layer])
            gu = F.linear(h, self.w_gate_up[layer])
            x = x + F.linear(F.silu(gu[:, : cfg.ffn]) * gu[:, cfg.ffn:], self.w_down[layer])
        last = self._norm(x[meta.last_token_ix.to(self.device).long()], self.ln_final)
        if self.head32 is not None:
            return F.linear(last.float(), self.head32)
        return F.linear(last, self.embed).float()

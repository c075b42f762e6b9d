"""Plain-PyTorch restatement of futon's encoder forward (a parity checker).

Follows native/model.go:346-769 operation by operation (post-LN blocks,
NeoX RoPE from f64-built tables, exact-erf GELU, SwiGLU, CLS/mean pooling,
matryoshka LayerNorm, L2) and the Q8 scheme of native/quant.go, in float32
(or float64) with TF32 disabled. It is pinned against the CPU oracle at
small sizes (tests/test_torch_ref.py) and then checks the CUDA path at full
benchmark sizes, where the scalar oracle would take minutes.
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import numpy as np
import torch


def _q8_rows(x: torch.Tensor):
    """quantizeRowQ8 (quant.go:42-70) per row, in float64."""
    amax = x.abs().amax(dim=1)
    scale = (amax / 127.0).to(torch.float32)  # f32 division
    inv = torch.where(amax > 0, 127.0 / amax.double(), torch.zeros_like(amax, dtype=torch.float64))
    v = x.double() * inv[:, None]
    q = torch.sign(v) * torch.floor(v.abs() + 0.5)  # round half away from zero
    q = q.clamp(-127, 127)
    return q, scale


def q8_matmul(a: torch.Tensor, qb: torch.Tensor, sb: torch.Tensor, bias: Optional[torch.Tensor]):
    qa, sa = _q8_rows(a.float())
    acc = qa @ qb.double().t()  # exact: |sum| < 2^53
    out = acc.float() * (sa[:, None] * sb[None, :])
    if bias is not None:
        out = out + bias
    return out


class TorchRef:
    def __init__(self, cfg, tensors: Dict[str, np.ndarray], device="cpu", dtype=torch.float32,
                 q8: bool = False):
        self.cfg, self.dev, self.dt, self.q8 = cfg, torch.device(device), dtype, q8
        self.t = {k: torch.as_tensor(np.array(v, dtype=np.float32)).to(self.dev, dtype)
                  for k, v in tensors.items()}
        self.qw = {}
        if q8:
            for k, v in self.t.items():
                if k.startswith("layers.") and k.endswith(".weight") and "norm" not in k:
                    q, s = _q8_rows(v.float())
                    self.qw[k] = (q, s)
        h, H = cfg.hidden_size, cfg.num_heads
        self.hd = h // H
        if cfg.position_encoding == "rope":
            ms, half = cfg.effective_max_seq_len(), self.hd // 2
            t = np.arange(ms, dtype=np.float64)[:, None]
            i = np.arange(half, dtype=np.float64)[None, :]
            freq = 1.0 / np.power(cfg.rope_theta, (2 * i) / self.hd)
            ang = t * freq
            self.cos = torch.as_tensor(np.cos(ang).astype(np.float32)).to(self.dev, dtype)
            self.sin = torch.as_tensor(np.sin(ang).astype(np.float32)).to(self.dev, dtype)

    def _mm(self, x, name, bias_name):
        b = self.t.get(bias_name)
        if self.q8:
            q, s = self.qw[name]
            return q8_matmul(x, q, s, None if b is None else b.float()).to(self.dt)
        y = x @ self.t[name].t()
        return y + b if b is not None else y

    def _ln(self, x, w, b, eps):
        xd = x.double()
        mean = xd.mean(dim=-1, keepdim=True)
        var = ((xd - mean) ** 2).mean(dim=-1, keepdim=True)
        inv = (1.0 / torch.sqrt(var + float(np.float32(eps)))).to(self.dt)
        y = (x - mean.to(self.dt)) * inv
        if w is not None:
            y = y * w + b
        return y

    def _rot(self, x, L):
        half = self.hd // 2
        c, s = self.cos[:L][:, None, :], self.sin[:L][:, None, :]
        x1, x2 = x[..., :half], x[..., half:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)

    @torch.no_grad()
    def encode(self, ids, out_dim: int = 0) -> np.ndarray:
        cfg, t = self.cfg, self.t
        h, H, hd = cfg.hidden_size, cfg.num_heads, self.hd
        ids_t = torch.as_tensor(np.asarray(ids, dtype=np.int64), device=self.dev)
        L = ids_t.numel()
        x = t["embeddings.word"][ids_t]
        if cfg.type_vocab_size > 0:
            x = x + t["embeddings.token_type"][0]
        if cfg.position_encoding == "absolute":
            x = x + t["embeddings.position"][:L]
        eps = cfg.layer_norm_eps
        x = self._ln(x, t["embeddings.norm.weight"], t["embeddings.norm.bias"], eps)
        scale = 1.0 / math.sqrt(hd)
        for li in range(cfg.num_layers):
            p = f"layers.{li}."
            qkv = self._mm(x, p + "attn.qkv.weight", p + "attn.qkv.bias")
            q = qkv[:, :h].reshape(L, H, hd)
            k = qkv[:, h:2 * h].reshape(L, H, hd)
            v = qkv[:, 2 * h:].reshape(L, H, hd)
            if cfg.position_encoding == "rope":
                q, k = self._rot(q, L), self._rot(k, L)
            s = torch.einsum("qhd,khd->hqk", q, k) * scale
            pr = torch.softmax(s.double(), dim=-1).to(self.dt)
            o = torch.einsum("hqk,khd->qhd", pr, v).reshape(L, h)
            a = self._mm(o, p + "attn.out.weight", p + "attn.out.bias") + x
            x = self._ln(a, t[p + "norm1.weight"], t[p + "norm1.bias"], eps)
            f = self._mm(x, p + "mlp.fc1.weight", p + "mlp.fc1.bias")
            if cfg.activation == "swiglu":
                g = self._mm(x, p + "mlp.gate.weight", p + "mlp.gate.bias")
                f = f * (g * torch.sigmoid(g))
            else:
                f = 0.5 * f * (1.0 + torch.erf(f / math.sqrt(2.0)))
            y = self._mm(f, p + "mlp.fc2.weight", p + "mlp.fc2.bias") + x
            x = self._ln(y, t[p + "norm2.weight"], t[p + "norm2.bias"], eps)
        pooled = x[0] if cfg.pooling == "cls" else x.sum(dim=0) * (1.0 / L)
        if out_dim and out_dim != h:
            if cfg.matryoshka is not None and cfg.matryoshka.layernorm:
                pooled = self._ln(pooled[None, :], None, None, 1e-5)[0]
            pooled = pooled[:out_dim]
        if cfg.normalize:
            ss = (pooled.double() ** 2).sum()
            if ss > 0:
                pooled = pooled * (1.0 / torch.sqrt(ss)).to(self.dt)
        return pooled.float().cpu().numpy()

    def encode_packed(self, ids, cu, out_dim: int = 0) -> np.ndarray:
        return np.stack([self.encode(ids[cu[i]:cu[i + 1]], out_dim) for i in range(len(cu) - 1)])

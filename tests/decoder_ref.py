"""fp32 torch restatement of the tensor-parallel decoder's math (TP = 1) for the
decoder tests: dequantised weights from the oracle, explicit sink + window
attention over the full key history, no library kernels.  The fused q|k|v and
gate|up linears are evaluated as one product and split (their LoRA B is
block-diagonal, so each part equals its own linear)."""

from __future__ import annotations

import math

import numpy as np
import torch

from oracle import dequantize_gptq


def _dense(lin, device):
    W = dequantize_gptq(lin.qweight.cpu().numpy(), lin.scales.cpu().numpy(), lin.qzeros.cpu().numpy(),
                        lin.group)
    A = lin.lora_A.float().to(device)
    B = lin.lora_B.float().to(device)
    return torch.from_numpy(np.asarray(W, dtype=np.float32)).to(device), A, B, float(lin.lora_scale)


class RefDecoder:
    def __init__(self, dec):
        self.cfg, self.dev = dec.cfg, dec.device
        f = lambda t: t.float()
        self.embed, self.lm_head, self.final_norm = f(dec.embed), f(dec.lm_head), f(dec.final_norm)
        self.layers = []
        for L in dec.layers:
            R = {k: f(L[k]) for k in ("in_norm", "post_norm", "q_norm", "k_norm")}
            for k in ("qkv", "o", "gate_up", "down"):
                R[k] = _dense(L[k], self.dev)
            R["qkv_splits"], R["gate_up_splits"] = L["qkv"].splits, L["gate_up"].splits
            R["gate_up_il"] = getattr(L["gate_up"], "interleaved", False)
            self.layers.append(R)
        self.cos, self.sin = dec.cos, dec.sin
        self.hq, self.hkv = dec.hq, dec.hkv
        self.kh = [[] for _ in dec.layers]  # per layer: list of (pos, k [B, hkv, D], v)
        self.count = 0

    def _rms(self, x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.rms_eps) * w

    @staticmethod
    def _lin(x, p):
        W, A, B, s = p
        return x @ W + s * ((x @ A) @ B)

    def _rope(self, x, pos):
        D = x.size(-1)
        c, s = self.cos[pos], self.sin[pos]
        rot = torch.cat([-x[..., D // 2:], x[..., :D // 2]], dim=-1)
        return x * c + rot * s

    def token(self, tok: torch.Tensor):
        """one position for every sequence: tok [B] -> hidden [B, H] (before the final norm)"""
        cfg = self.cfg
        p = self.count
        x = self.embed[tok]
        B, D = x.size(0), cfg.head_dim
        for li, L in enumerate(self.layers):
            h = self._rms(x, L["in_norm"])
            q_, k_, v_ = self._lin(h, L["qkv"]).split(L["qkv_splits"], dim=-1)
            q = self._rms(q_.reshape(B, self.hq, D), L["q_norm"])
            k = self._rms(k_.reshape(B, self.hkv, D), L["k_norm"])
            v = v_.reshape(B, self.hkv, D)
            q, k = self._rope(q, p), self._rope(k, p)
            self.kh[li].append((p, k, v))
            keep = [(kp, kk, vv) for kp, kk, vv in self.kh[li]
                    if kp < cfg.sink or p - cfg.window < kp <= p]
            K = torch.stack([e[1] for e in keep], dim=1)  # [B, L, hkv, D]
            V = torch.stack([e[2] for e in keep], dim=1)
            rep = self.hq // self.hkv
            K = K.repeat_interleave(rep, dim=2)
            V = V.repeat_interleave(rep, dim=2)
            sc = torch.einsum("bhd,blhd->bhl", q, K) / math.sqrt(D)
            a = torch.einsum("bhl,blhd->bhd", sc.softmax(-1), V).reshape(B, self.hq * D)
            x = x + self._lin(a, L["o"])
            h = self._rms(x, L["post_norm"])
            gu = self._lin(h, L["gate_up"])
            if L["gate_up_il"]:  # blocks of 8 gate then 8 up columns
                inter = L["gate_up_splits"][0]
                gu = gu.view(B, inter // 8, 2, 8).transpose(1, 2).reshape(B, 2 * inter)
            g, u = gu.split(L["gate_up_splits"], dim=-1)
            x = x + self._lin(g * torch.sigmoid(g) * u, L["down"])
        self.count += 1
        return x

    def logits(self, x):
        return self._rms(x, self.final_norm) @ self.lm_head

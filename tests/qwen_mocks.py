"""Stand-ins for the third-party modules patch_qwen reads: a GPTQ
``QuantLinear`` (attributes ``qweight``, ``scales``, ``qzeros``,
``group_size``) and a PEFT LoRA wrapper (``base_layer``,
``lora_A["default"]``, ``lora_B["default"]``, ``lora_alpha["default"]``),
plus a tiny HF Qwen3 model whose projections use them.  Neither peft nor a
GPTQ package is installed; these mocks expose the attribute names the
reference reads (``qextract/patch.py:117-148``) and compute the reference
math in torch fp32.
"""

from __future__ import annotations

import numpy as np
import torch
from torch import nn


def dequant_torch(qweight, scales, qzeros, group, g_idx=None):
    K8, N = qweight.shape
    shifts = torch.arange(8, device=qweight.device, dtype=torch.int32) * 4
    q = (qweight.unsqueeze(1) >> shifts.view(1, 8, 1)) & 0xF  # [K/8, 8, N]
    q = q.reshape(K8 * 8, N).float()
    z = (qzeros.unsqueeze(2) >> shifts.view(1, 1, 8)) & 0xF  # [G, N/8, 8]
    z = z.reshape(qzeros.size(0), N).float()
    g = torch.arange(K8 * 8, device=qweight.device) // group if g_idx is None else g_idx.long()
    return ((q - z[g]) * scales.float()[g]).half()


class MockQuantLinear(nn.Module):
    """``act_order``: a GPTQ act-order layer, whose ``g_idx`` assigns the input
    rows to the groups in a shuffled order (each group still holds ``group``
    rows), with random zero points."""

    def __init__(self, K, N, group=128, seed=0, act_order=False):
        super().__init__()
        rng = np.random.default_rng(seed)
        qw = rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.uint64).astype(np.uint32).view(np.int32)
        sc = rng.uniform(0.005, 0.02, size=(K // group, N)).astype(np.float16)
        zn = np.full((K // group, N // 8), 0x88888888, dtype=np.uint32).view(np.int32)
        if act_order:
            zn = rng.integers(0, 2 ** 32, size=zn.shape, dtype=np.uint64).astype(np.uint32).view(np.int32)
            self.register_buffer("g_idx", torch.from_numpy(
                rng.permutation(np.arange(K) // group).astype(np.int32)))
        self.register_buffer("qweight", torch.from_numpy(qw))
        self.register_buffer("scales", torch.from_numpy(sc))
        self.register_buffer("qzeros", torch.from_numpy(zn))
        self.group_size = group
        self.in_features, self.out_features = K, N
        self.bias = None

    def forward(self, x):
        w = dequant_torch(self.qweight, self.scales, self.qzeros, self.group_size,
                          getattr(self, "g_idx", None))
        return (x.float() @ w.float()).to(x.dtype)


class MockLoraLinear(nn.Module):
    def __init__(self, K, N, r=16, alpha=32.0, group=128, seed=0, act_order=False):
        super().__init__()
        self.base_layer = MockQuantLinear(K, N, group, seed, act_order)
        g = torch.Generator().manual_seed(seed + 1)
        a = nn.Linear(K, r, bias=False)
        b = nn.Linear(r, N, bias=False)
        with torch.no_grad():
            a.weight.copy_(torch.randn(r, K, generator=g) * 0.02)
            b.weight.copy_(torch.randn(N, r, generator=g) * 0.02)
        self.lora_A = nn.ModuleDict({"default": a})
        self.lora_B = nn.ModuleDict({"default": b})
        self.lora_alpha = {"default": alpha}
        self.r = {"default": r}

    def forward(self, x):
        base = self.base_layer(x).float()
        A = self.lora_A["default"].weight.float()
        B = self.lora_B["default"].weight.float()
        lora = (x.float() @ A.t()) @ B.t()
        r = A.shape[0]
        return (base + (self.lora_alpha["default"] / r) * lora).to(x.dtype)


def make_tiny_qwen3(num_layers=2, hidden=256, inter=512, heads=4, kv_heads=2, head_dim=64,
                    vocab=512, lora=True, seed=0, act_order=False):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter,
                      num_hidden_layers=num_layers, num_attention_heads=heads,
                      num_key_value_heads=kv_heads, head_dim=head_dim, max_position_embeddings=4096,
                      rope_theta=1e6, rms_norm_eps=1e-6, tie_word_embeddings=False)
    cfg._attn_implementation = "eager"
    torch.manual_seed(seed)
    model = Qwen3ForCausalLM(cfg)
    s = seed * 100
    for layer in model.model.layers:
        at, mlp = layer.self_attn, layer.mlp
        shapes = {"q_proj": (hidden, heads * head_dim), "k_proj": (hidden, kv_heads * head_dim),
                  "v_proj": (hidden, kv_heads * head_dim), "o_proj": (heads * head_dim, hidden),
                  "gate_proj": (hidden, inter), "up_proj": (hidden, inter),
                  "down_proj": (inter, hidden)}
        for name, (K, N) in shapes.items():
            parent = at if name in ("q_proj", "k_proj", "v_proj", "o_proj") else mlp
            s += 1
            mod = (MockLoraLinear(K, N, seed=s, act_order=act_order) if lora
                   else MockQuantLinear(K, N, seed=s, act_order=act_order))
            setattr(parent, name, mod)
        with torch.no_grad():
            layer.input_layernorm.weight.normal_(1.0, 0.1)
            layer.post_attention_layernorm.weight.normal_(1.0, 0.1)
    return model

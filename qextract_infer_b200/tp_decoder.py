"""Tensor-parallel Qwen3-architecture decoder on this library's operators.

The model the reference patches (``qextract/patch.py:10-70``: HF Qwen3 with
GPTQ int4 linears and PEFT LoRA adapters) written directly against the
operators, sharded over ``torch.distributed`` ranks (one process per GPU,
NCCL):

* column-parallel q / k / v / gate / up: each rank holds N / tp output columns
  (their scales, qzeros and LoRA B columns; LoRA A replicated);
* row-parallel o / down: each rank holds K / tp input rows (LoRA A rows split,
  LoRA B replicated), so the partial products and the LoRA partials meet in
  one all-reduce after o and one after down;
* q heads 32 / tp and KV heads 8 / tp per rank, each rank with its own
  StreamingLLM ring (sink + window) for its KV heads;
* embeddings replicated, the fp16 lm_head split over the vocabulary, greedy
  sampling by an all-gather of the per-rank (max, argmax).

The projections that read the same input are fused: q|k|v and gate|up are
each one W4A16-LoRA call (weights side by side, LoRA A side by side, LoRA B
block-diagonal, rank zero-padded to a supported size: the same math).  Per
decode step and layer (7 launches at one or two sequences, 8 beyond): qkv GEMV
-> per-head RMSNorm of q and k (Qwen3), RoPE (theta 1e6, keys stored post-RoPE
at their absolute positions), the ring append and the GQA decode attention over
sink + window (including the new token), in one kernel or as append + attention
-> o GEMV -> all-reduce + residual add + RMSNorm in
one kernel -> gate|up GEMV with the SwiGLU epilogue (gate and up columns
interleaved in blocks of 8, so one CTA holds both halves of an output) -> down
GEMV -> all-reduce + residual add + the next RMSNorm in one kernel.  With more than one rank the all-reduce is a
one-shot exchange over NVLink peer memory inside that kernel
(``nvlink_allreduce.py``); prefill chunks all-reduce with NCCL.  Prefill chunks
run the same projections with the tensor-core GEMM; their attention (each
query over the sinks, the previous window and the causal part of its chunk)
is ``prefill_attention``, which reads the ring in place.

Weights are synthetic: every full tensor comes from a generator seeded by
(seed, layer, projection) on the device and each rank keeps its shard, so the
model is the same for every tensor-parallel size.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from . import _C
from .tp_shard import merge_greedy, shard_quant_linear, shard_vocab


@dataclass
class DecoderConfig:
    num_layers: int = 36
    hidden: int = 4096
    intermediate: int = 12288
    num_q_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    vocab: int = 151936
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    lora_rank: int = 16
    lora_alpha: float = 32.0  # alpha / r = 2
    group_size: int = 128
    sink: int = 4
    window: int = 4092
    init_std: float = 0.02  # embeddings, norms, lm_head ~ N(0, std)


class ShardedQuantLinear:
    """One rank's shard of a GPTQ int4 (group-wise, packed qzeros all 8) + LoRA
    linear; ``split`` is "col" (N), "row" (K) or None (replicated)."""

    def __init__(self, K: int, N: int, cfg: DecoderConfig, seed: int, device, rank: int, world: int,
                 split: str | None):
        G, r = cfg.group_size, cfg.lora_rank
        g = torch.Generator(device=device).manual_seed(seed)
        qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=g, device=device,
                           dtype=torch.int32)
        sc = (torch.rand(K // G, N, generator=g, device=device) * 0.015 + 0.005).half()
        A = (torch.randn(K, r, generator=g, device=device) * 0.02).half()
        B = (torch.randn(r, N, generator=g, device=device) * 0.02).half()
        qz = torch.full((K // G, N // 8), 0x88888888 - 2 ** 32, dtype=torch.int32, device=device)
        qw, sc, qz, A, B = shard_quant_linear(qw, sc, qz, A, B, split, rank, world, G)
        self.K, self.N = qw.size(0) * 8, qw.size(1)
        self.qweight, self.scales, self.qzeros = qw.contiguous(), sc.contiguous(), qz.contiguous()
        self.lora_A, self.lora_B = A.contiguous(), B.contiguous()
        self.group = G
        self.lora_scale = float(np.float32(cfg.lora_alpha) / np.float32(r))  # alpha / r in fp32

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return _C._w4a16(x, self.qweight, self.scales, self.qzeros, self.lora_A, self.lora_B,
                         self.group, self.lora_scale, 0)

    def weight_bytes(self) -> int:
        """bytes of the operands one call reads (int4 weights, scales, qzeros, LoRA A and B)"""
        return sum(t.numel() * t.element_size()
                   for t in (self.qweight, self.scales, self.qzeros, self.lora_A, self.lora_B))


class FusedQuantLinear:
    """Column-parallel linears that read the same input, as one W4A16-LoRA
    call: qweight / scales / qzeros side by side along N, LoRA A side by side
    and LoRA B block-diagonal, the rank zero-padded to ``rank`` (the padding
    contributes 0, so every part's output equals its own linear's).  The parts
    share alpha / r."""

    def __init__(self, parts: list, rank: int):
        dev = parts[0].qweight.device
        self.K = parts[0].K
        self.splits = [p.N for p in parts]
        self.N = sum(self.splits)
        self.qweight = torch.cat([p.qweight for p in parts], 1).contiguous()
        self.scales = torch.cat([p.scales for p in parts], 1).contiguous()
        self.qzeros = torch.cat([p.qzeros for p in parts], 1).contiguous()
        rs = [p.lora_A.size(1) for p in parts]
        if sum(rs) > rank or len({p.lora_scale for p in parts}) != 1:
            raise ValueError("fused parts need one alpha / r and a total rank <= rank")
        A = torch.zeros(self.K, rank, dtype=torch.float16, device=dev)
        B = torch.zeros(rank, self.N, dtype=torch.float16, device=dev)
        r0 = n0 = 0
        for p, r in zip(parts, rs):
            A[:, r0:r0 + r] = p.lora_A
            B[r0:r0 + r, n0:n0 + p.N] = p.lora_B
            r0, n0 = r0 + r, n0 + p.N
        self.lora_A, self.lora_B = A, B
        self.group, self.lora_scale = parts[0].group, parts[0].lora_scale
        self._bytes = sum(p.weight_bytes() for p in parts)  # the parts' own operands (no padding)

    def weight_bytes(self) -> int:
        """algorithmic bytes of one call: the parts' operands (the zero padding of
        the fused LoRA factors is not counted)"""
        return self._bytes

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return _C._w4a16(x, self.qweight, self.scales, self.qzeros, self.lora_A, self.lora_B,
                         self.group, self.lora_scale, 0)

    def addnorm(self, res: torch.Tensor, delta: torch.Tensor, norm_w: torch.Tensor, eps: float,
                res_out: torch.Tensor, swiglu: bool = False) -> torch.Tensor:
        """``res_out = res + delta``, then this projection (its SwiGLU form with
        ``swiglu``) of ``rmsnorm(res_out) * norm_w``: one launch (decode rows)."""
        return _C._w4a16_addnorm(res, delta, norm_w, eps, res_out, self.qweight, self.scales, self.qzeros,
                                 self.lora_A, self.lora_B, self.group, self.lora_scale, 0, swiglu)

    def interleave_gate_up(self) -> "FusedQuantLinear":
        """Reorders a fused [gate | up] pair into blocks of 8 gate and 8 up
        columns (``_C.interleave_gate_up``) for ``swiglu``; ``__call__`` then
        returns the reordered columns."""
        inter = self.splits[0]
        if len(self.splits) != 2 or self.splits[1] != inter:
            raise ValueError("interleave_gate_up needs two parts of equal width")
        il = _C.interleave_gate_up
        self.qweight, self.scales = il(self.qweight, inter), il(self.scales, inter)
        self.qzeros = il(self.qzeros, inter, packed=True)
        self.lora_B = il(self.lora_B, inter)
        self.interleaved = True
        return self

    def swiglu(self, x: torch.Tensor) -> torch.Tensor:
        """silu(gate) * up of the interleaved gate|up pair: one launch for
        decode rows (the GEMV's SwiGLU epilogue)"""
        return _C._w4a16_swiglu(x, self.qweight, self.scales, self.qzeros, self.lora_A, self.lora_B,
                                self.group, self.lora_scale, 0)


def _padded_rank(r: int) -> int:
    """smallest LoRA rank the kernels take that holds r"""
    for s in (8, 16, 32, 48, 64, 128):
        if s >= r:
            return s
    raise ValueError(f"fused LoRA rank {r} > 128")


class TPDecoder:
    def __init__(self, cfg: DecoderConfig, batch: int, device, seed: int = 4,
                 group: dist.ProcessGroup | None = None, nvlink_allreduce: bool = True):
        self.cfg, self.batch, self.device = cfg, batch, torch.device(device)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        w, r = self.world, self.rank
        if cfg.num_q_heads % w or cfg.num_kv_heads % w or cfg.intermediate % w or cfg.vocab % w:
            raise ValueError(f"tensor-parallel size {w} does not divide the heads / sizes")
        self.hq, self.hkv = cfg.num_q_heads // w, cfg.num_kv_heads // w
        D, H = cfg.head_dim, cfg.hidden
        dev = self.device
        gen = torch.Generator(device=dev)

        def normal(shape, s):
            gen.manual_seed(s)
            return (torch.randn(*shape, generator=gen, device=dev) * cfg.init_std).half()

        self.embed = normal((cfg.vocab, H), seed * 1000003 + 1)
        self.lm_head = shard_vocab(normal((H, cfg.vocab), seed * 1000003 + 2), r, w).contiguous()
        self.final_norm = normal((H,), seed * 1000003 + 3)
        self.layers = []
        for li in range(cfg.num_layers):
            base = seed * 1000003 + 100 + li * 16
            q = ShardedQuantLinear(H, cfg.num_q_heads * D, cfg, base + 4, dev, r, w, "col")
            k = ShardedQuantLinear(H, cfg.num_kv_heads * D, cfg, base + 5, dev, r, w, "col")
            v = ShardedQuantLinear(H, cfg.num_kv_heads * D, cfg, base + 6, dev, r, w, "col")
            gate = ShardedQuantLinear(H, cfg.intermediate, cfg, base + 8, dev, r, w, "col")
            up = ShardedQuantLinear(H, cfg.intermediate, cfg, base + 9, dev, r, w, "col")
            L = dict(
                in_norm=normal((H,), base), post_norm=normal((H,), base + 1),
                q_norm=normal((D,), base + 2), k_norm=normal((D,), base + 3),
                qkv=FusedQuantLinear([q, k, v], _padded_rank(3 * cfg.lora_rank)),
                o=ShardedQuantLinear(cfg.num_q_heads * D, H, cfg, base + 7, dev, r, w, "row"),
                gate_up=FusedQuantLinear([gate, up], _padded_rank(2 * cfg.lora_rank)).interleave_gate_up(),
                down=ShardedQuantLinear(cfg.intermediate, H, cfg, base + 10, dev, r, w, "row"),
            )
            del q, k, v, gate, up
            self.layers.append(L)
        self.cache = _C.RingBufferKVCache(cfg.num_layers, self.hkv, D, cfg.sink, cfg.window,
                                          batch=batch, device=dev)
        # q/k norm + RoPE + append fused into the attention kernel for a few
        # sequences (one launch fewer per layer, same time); for many, the
        # separate append kernel is faster (32 sequences: 86 vs 96 us per layer)
        self.fused_attention = batch * self.hkv <= 16
        self.max_pos = 1 << 16
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D))
        ang = torch.arange(self.max_pos, device=dev, dtype=torch.float32)[:, None] * inv[None, :]
        self.cos = torch.cat([ang.cos(), ang.cos()], dim=-1)  # [pos, D]
        self.sin = torch.cat([ang.sin(), ang.sin()], dim=-1)
        # decode steps (batch rows) all-reduce through NVLink peer memory fused with the
        # residual add and RMSNorm; prefill chunks use NCCL
        self.ar = None
        if self.world > 1 and nvlink_allreduce:
            from .nvlink_allreduce import NVLinkAllReduce
            self.ar = NVLinkAllReduce(group if group is not None else dist.group.WORLD, batch, H, dev)

    def check_device_error(self) -> None:
        """Raise if a bounded wait inside one of this rank's kernels ran out
        (a peer that did not arrive, a stalled copy): the tokens of the steps
        since the last check are then undefined.  Synchronises the device."""
        with torch.cuda.device(self.device):
            _C.check_device_error(f"tensor-parallel decoder rank {self.rank}")

    def close(self) -> None:
        """release the NVLink all-reduce buffers (collective: call on every rank)"""
        if self.ar is not None:
            self.ar.close()
            self.ar = None

    # ------------------------------------------------------------------ pieces
    def _allreduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def _reduce_add_norm(self, partial: torch.Tensor, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """x += all_reduce(partial) in place; returns rmsnorm(x) * w"""
        if self.ar is not None:
            return self.ar.add_rmsnorm(partial, x, w, self.cfg.rms_eps)
        return _C.add_rmsnorm(x, self._allreduce(partial), w, self.cfg.rms_eps)

    def _rope(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        """x [..., T, heads, D] fp16; cos/sin [T, D] fp32 -> rotated fp16 (HF rotate_half)."""
        xf = x.float()
        half = x.size(-1) // 2
        rot = torch.cat([-xf[..., half:], xf[..., :half]], dim=-1)
        return (xf * cos[:, None, :] + rot * sin[:, None, :]).half()

    def _head_norm(self, t: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        return _C.fused_rmsnorm(t.contiguous(), w, self.cfg.rms_eps)

    def _mlp(self, L, h: torch.Tensor) -> torch.Tensor:
        return self._allreduce(L["down"](L["gate_up"].swiglu(h)))

    # ------------------------------------------------------------------ decode
    def decode_step(self, tokens: torch.Tensor, return_hidden: bool = False):
        """One greedy step for the batch: ``tokens`` int64 [B] (device) -> next
        tokens int64 [B] (and the final hidden state [B, H] if asked).  The
        position is the cache's token count."""
        cfg, B, D = self.cfg, self.batch, self.cfg.head_dim
        eps = cfg.rms_eps
        pos = self.cache.get_total_written()
        cos, sin = self.cos[pos], self.sin[pos]
        x = self.embed.index_select(0, tokens)  # [B, H], the residual stream
        h = _C.fused_rmsnorm(x, self.layers[0]["in_norm"], eps)
        n = len(self.layers)
        # one GPU and a few rows: the residual add + RMSNorm before the MLP and
        # before the next layer's q|k|v run as those projections' prologue (5
        # launches per layer); the residual alternates between two buffers
        fuse = self.world == 1 and B <= 8
        xo = torch.empty_like(x) if fuse else None
        dn = None
        for li, L in enumerate(self.layers):
            if fuse and li > 0:
                qkv = L["qkv"].addnorm(x, dn, L["in_norm"], eps, xo)  # x + down of the layer before
                x, xo = xo, x
            else:
                qkv = L["qkv"](h)
            if self.fused_attention:
                att = _C.decode_attention_qkv(qkv, self.hq, self.hkv, L["q_norm"], L["k_norm"], eps,
                                              cos, sin, self.cache.k[li], self.cache.v[li], cfg.sink,
                                              cfg.window, pos)
            else:
                q = _C.qk_norm_rope_append(qkv, self.hq, self.hkv, L["q_norm"], L["k_norm"], eps, cos,
                                           sin, self.cache.k[li], self.cache.v[li], cfg.sink, cfg.window,
                                           pos)
                att = _C.decode_attention(q, self.cache.k[li], self.cache.v[li], pos + 1, cfg.sink,
                                          cfg.window, after_append=True)
            o = L["o"](att.view(B, self.hq * D))
            if fuse:
                gu = L["gate_up"].addnorm(x, o, L["post_norm"], eps, xo, swiglu=True)  # x + o
                x, xo = xo, x
                dn = L["down"](gu)
                if li + 1 == n:
                    h = _C.add_rmsnorm(x, dn, self.final_norm, eps)  # x += down; the final RMSNorm
                continue
            h = self._reduce_add_norm(o, x, L["post_norm"])  # x += o
            dn = L["down"](L["gate_up"].swiglu(h))
            nxt_w = self.layers[li + 1]["in_norm"] if li + 1 < n else self.final_norm
            h = self._reduce_add_norm(dn, x, nxt_w)  # x += down; the next RMSNorm
        self.cache.advance(1)
        nxt = self._greedy_normed(h)
        return (nxt, x) if return_hidden else nxt

    def _greedy_logits(self, x: torch.Tensor) -> torch.Tensor:
        """this rank's vocabulary slice of the logits [B, V / tp] (fp16; tests only)"""
        h = _C.fused_rmsnorm(x, self.final_norm, self.cfg.rms_eps)
        return h @ self.lm_head

    def _greedy(self, x: torch.Tensor) -> torch.Tensor:
        return self._greedy_normed(_C.fused_rmsnorm(x, self.final_norm, self.cfg.rms_eps))

    def _greedy_normed(self, h: torch.Tensor) -> torch.Tensor:
        """greedy tokens from the final-normed hidden state"""
        val, idx = _C.lm_head_argmax(h, self.lm_head, self.rank * self.lm_head.size(1))
        if self.world > 1:
            vals = [torch.empty_like(val) for _ in range(self.world)]
            idxs = [torch.empty_like(idx) for _ in range(self.world)]
            dist.all_gather(vals, val, group=self.group)
            dist.all_gather(idxs, idx, group=self.group)
            idx = merge_greedy(torch.stack(vals), torch.stack(idxs))  # [world, B] -> [B]
        return idx

    # ----------------------------------------------------------------- prefill
    def prefill(self, tokens: torch.Tensor, chunk: int = 2048, return_hidden: bool = False):
        """``tokens`` int64 [B, T] (device); returns the greedy next tokens [B]
        (and the last position's hidden state [B, H] if asked)."""
        cfg, B, D = self.cfg, self.batch, self.cfg.head_dim
        T = tokens.size(1)
        x_last = None
        for t0 in range(0, T, chunk):
            tc = tokens[:, t0:t0 + chunk]
            n = tc.size(1)
            c = self.cache.get_total_written()
            cos, sin = self.cos[c:c + n], self.sin[c:c + n]
            x = self.embed.index_select(0, tc.reshape(-1)).view(B * n, cfg.hidden)
            for li, L in enumerate(self.layers):
                h = _C.fused_rmsnorm(x, L["in_norm"], cfg.rms_eps)
                qp, kp, vp = L["qkv"](h).split(L["qkv"].splits, dim=-1)
                q = self._head_norm(qp.reshape(B * n * self.hq, D), L["q_norm"])
                k = self._head_norm(kp.reshape(B * n * self.hkv, D), L["k_norm"])
                v = vp.reshape(B, n, self.hkv, D).contiguous()
                q = self._rope(q.view(B, n, self.hq, D), cos, sin)
                k = self._rope(k.view(B, n, self.hkv, D), cos, sin)
                # the chunk over the ring (read in place) and its own keys, then the append
                att = _C.prefill_attention(q, k.contiguous(), v, self.cache.k[li], self.cache.v[li], c,
                                           cfg.sink, cfg.window)  # [B, n, hq, D]
                self.cache.append(k, v, li)
                att = att.reshape(B * n, self.hq * D)
                x = x + self._allreduce(L["o"](att))
                h = _C.fused_rmsnorm(x, L["post_norm"], cfg.rms_eps)
                x = x + self._mlp(L, h)
            x_last = x.view(B, n, cfg.hidden)[:, -1].contiguous()
        nxt = self._greedy(x_last)
        return (nxt, x_last) if return_hidden else nxt

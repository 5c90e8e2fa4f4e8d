"""One gloo rank of the tensor-parallel sharding check (CPU, no GPU).

Every rank builds the same full weights of one small Qwen3-shaped decoder
layer (seeded numpy), takes its shard with the decoder's own sharding rules
(``qextract_infer_b200.tp_shard``), computes its part with the numpy oracle
and exchanges over ``gloo`` exactly where the decoder exchanges over NCCL /
NVLink: an all-gather of column-parallel outputs (here only to compare them),
an all-reduce of the row-parallel partials (base and LoRA together) after o
and after down, and an all-gather of (max, index) for the vocabulary-split
greedy step.  Every rank compares with the unsharded oracle.
"""

from __future__ import annotations

import datetime
import os

import numpy as np
import torch
import torch.distributed as dist

from oracle import gqa_decode_attention_ref, make_gemv_inputs, rmsnorm_ref, swiglu_ref_single_round
from oracle import w4a16_lora_gemv_ref
from qextract_infer_b200.tp_shard import merge_greedy, shard_quant_linear, shard_vocab

# a config[4]-shaped layer at small sizes: hidden 512, 8 q / 4 kv heads of 64,
# intermediate 1024, group 128, LoRA r16 alpha/r 2, vocabulary 1024
H, I, HQ, HKV, D, G, R, ALPHA, V = 512, 1024, 8, 4, 64, 128, 16, 32.0, 1024
B, CTX = 3, 37   # batch rows, cached KV positions per sequence
TOL = 1e-2
# tp 8 needs 8 KV heads and o / down input slices of whole quantisation groups:
# a wider layer (hidden 1024, 16 q / 8 kv heads of 64, intermediate 2048)
WIDE = dict(H=1024, I=2048, HQ=16, HKV=8, D=64, V=1024)


def _linear(K, N, seed):
    d = make_gemv_inputs(1, K, N, R, group_size=G, seed=seed)
    rng = np.random.default_rng(seed + 1)
    # random zero points and larger LoRA factors so every term matters
    z = rng.integers(0, 16, size=(K // G, N)).astype(np.uint32).reshape(K // G, N // 8, 8)
    d["zeros"] = np.bitwise_or.reduce(z << (np.arange(8, dtype=np.uint32) * 4), axis=2).view(np.int32)
    d["lora_A"] = (rng.standard_normal((K, R)) * 0.1).astype(np.float16)
    d["lora_B"] = (rng.standard_normal((R, N)) * 0.1).astype(np.float16)
    return d


def _shard(d, split, rank, world):
    t = [torch.from_numpy(np.ascontiguousarray(d[k]))
         for k in ("qweight", "scales", "zeros", "lora_A", "lora_B")]
    return [x.contiguous().numpy() for x in shard_quant_linear(*t, split, rank, world, G)]


def _apply(x, shard, f32=False):
    qw, sc, qz, A, Bm = shard
    return w4a16_lora_gemv_ref(x, qw, sc, qz, A, Bm, G, ALPHA, return_f32=f32)


def _close(a, b, what, atol=TOL):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    bad = np.abs(a - b) > atol + TOL * np.abs(b)
    if bad.any():
        raise AssertionError(f"{what}: {bad.sum()} of {a.size} out of tolerance, "
                             f"max err {np.abs(a - b).max()}")


def _all_reduce_np(a):
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    dist.all_reduce(t)
    return t.numpy()


def _all_gather_cols(a):
    t = torch.from_numpy(np.ascontiguousarray(a))
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return torch.cat(out, dim=-1).numpy()


def run(rank: int, world: int, port: int) -> None:
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(port)
    if HKV % world:
        globals().update(WIDE)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        _check(rank, world)
    finally:
        dist.destroy_process_group()


def _check(rank: int, world: int) -> None:
    rng = np.random.default_rng(123)
    x = rng.standard_normal((B, H)).astype(np.float16)
    in_norm = (rng.standard_normal(H) * 0.1 + 1).astype(np.float16)
    post_norm = (rng.standard_normal(H) * 0.1 + 1).astype(np.float16)
    lm_head = rng.standard_normal((H, V)).astype(np.float16)
    kcache = rng.standard_normal((B, CTX, HKV, D)).astype(np.float16)
    vcache = rng.standard_normal((B, CTX, HKV, D)).astype(np.float16)
    W = {name: _linear(K, N, seed) for name, K, N, seed in (
        ("q", H, HQ * D, 11), ("k", H, HKV * D, 12), ("v", H, HKV * D, 13), ("o", HQ * D, H, 14),
        ("gate", H, I, 15), ("up", H, I, 16), ("down", I, H, 17))}
    hq, hkv = HQ // world, HKV // world

    # unsharded oracle
    h = rmsnorm_ref(x, in_norm)
    q_full = _apply(h, _shard(W["q"], None, 0, 1))
    att_full = np.stack([gqa_decode_attention_ref(q_full[b].reshape(HQ, D), kcache[b], vcache[b])
                         for b in range(B)]).reshape(B, HQ * D)
    o_full = _apply(att_full, _shard(W["o"], None, 0, 1), f32=True)
    x1 = (x.astype(np.float32) + o_full.astype(np.float16).astype(np.float32)).astype(np.float16)
    h1 = rmsnorm_ref(x1, post_norm)
    act_full = swiglu_ref_single_round(_apply(h1, _shard(W["gate"], None, 0, 1)),
                                       _apply(h1, _shard(W["up"], None, 0, 1)))
    dn_full = _apply(act_full, _shard(W["down"], None, 0, 1), f32=True)
    logits_full = h1.astype(np.float32) @ lm_head.astype(np.float32)

    # this rank: column-parallel q / k / v / gate / up
    cols = {n: _shard(W[n], "col", rank, world) for n in ("q", "k", "v", "gate", "up")}
    for n, N in (("q", HQ * D), ("k", HKV * D), ("v", HKV * D), ("gate", I), ("up", I)):
        assert cols[n][0].shape == (H // 8, N // world), (n, cols[n][0].shape)
        assert cols[n][2].shape == (H // G, N // world // 8)
        assert cols[n][3].shape == (H, R) and cols[n][4].shape == (R, N // world)
    q_i = _apply(h, cols["q"])
    k_i, v_i = _apply(h, cols["k"]), _apply(h, cols["v"])
    _close(_all_gather_cols(q_i), q_full, f"tp{world} q (column-parallel)")
    _close(_all_gather_cols(k_i), _apply(h, _shard(W["k"], None, 0, 1)), f"tp{world} k")
    _close(_all_gather_cols(v_i), _apply(h, _shard(W["v"], None, 0, 1)), f"tp{world} v")
    # this rank's heads: q heads [rank*hq, ...) read KV heads [rank*hkv, ...)
    kc, vc = kcache[:, :, rank * hkv:(rank + 1) * hkv], vcache[:, :, rank * hkv:(rank + 1) * hkv]
    att_i = np.stack([gqa_decode_attention_ref(q_i[b].reshape(hq, D), kc[b], vc[b])
                      for b in range(B)]).reshape(B, hq * D)
    _close(att_i, att_full[:, rank * hq * D:(rank + 1) * hq * D], f"tp{world} attention heads")

    # row-parallel o: partials (base + LoRA) summed by one all-reduce
    o_sh = _shard(W["o"], "row", rank, world)
    assert o_sh[0].shape == (HQ * D // 8 // world, H) and o_sh[3].shape == (HQ * D // world, R)
    assert o_sh[4].shape == (R, H)
    o_sum = _all_reduce_np(_apply(att_i, o_sh, f32=True))
    _close(o_sum, o_full, f"tp{world} o (row-parallel all-reduce)")
    x1_i = (x.astype(np.float32) + o_sum.astype(np.float16).astype(np.float32)).astype(np.float16)
    _close(x1_i, x1, f"tp{world} residual after o")
    h1_i = rmsnorm_ref(x1_i, post_norm)

    # MLP: column-parallel gate / up, SwiGLU on the rank's slice, row-parallel down
    act_i = swiglu_ref_single_round(_apply(h1_i, cols["gate"]), _apply(h1_i, cols["up"]))
    _close(act_i, act_full[:, rank * I // world:(rank + 1) * I // world], f"tp{world} SwiGLU slice")
    dn_sh = _shard(W["down"], "row", rank, world)
    # the row split alone: the rank's slice of the unsharded activations
    sl = slice(rank * I // world, (rank + 1) * I // world)
    dn_sum = _all_reduce_np(_apply(act_full[:, sl], dn_sh, f32=True))
    _close(dn_sum, dn_full, f"tp{world} down (row-parallel all-reduce)")
    # and from the rank's own SwiGLU slice, whose fp16 roundings after the o
    # all-reduce may differ by an ulp: the K-long sum carries them, so the bound
    # is relative to the output range
    dn_own = _all_reduce_np(_apply(act_i, dn_sh, f32=True))
    _close(dn_own, dn_full, f"tp{world} down from the rank's own activations",
           atol=TOL * float(np.abs(dn_full).max()))

    # vocabulary-split greedy
    lm_i = shard_vocab(torch.from_numpy(lm_head), rank, world).numpy()
    logits_i = torch.from_numpy(h1.astype(np.float32) @ lm_i.astype(np.float32))
    val, idx = logits_i.max(dim=-1)
    idx = idx + rank * (V // world)
    vals = [torch.empty_like(val) for _ in range(world)]
    idxs = [torch.empty_like(idx) for _ in range(world)]
    dist.all_gather(vals, val)
    dist.all_gather(idxs, idx)
    tok = merge_greedy(torch.stack(vals), torch.stack(idxs))
    ref_tok = torch.from_numpy(logits_full).argmax(dim=-1)
    assert torch.equal(tok, ref_tok), (tok, ref_tok)
    # ties go to the lowest rank (the first maximum of the full row)
    tv = torch.tensor([[1.0, 2.0], [1.0, 2.0]])
    ti = torch.tensor([[5, 7], [900, 901]])
    assert merge_greedy(tv, ti).tolist() == [5, 7]

"""Run under torchrun (one process per GPU): the tensor-parallel decoder on a
tiny Qwen3-shaped config against its fp32 restatement built from the full
(TP = 1) weights; every rank checks the final hidden state and the greedy
tokens after prefill and a few decode steps.  Exit status 0 = match."""

import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from qextract_infer_b200.tp_decoder import DecoderConfig, TPDecoder  # noqa: E402
from tests.decoder_ref import RefDecoder  # noqa: E402


def main():
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    world = dist.get_world_size()
    cfg = DecoderConfig(num_layers=2, hidden=512, intermediate=1024, num_q_heads=8, num_kv_heads=world,
                        head_dim=128, vocab=1024, sink=4, window=60, init_std=0.5)
    B, T = 2, 100
    dec = TPDecoder(cfg, batch=B, device=dev, seed=7)
    full = dec
    if world > 1:
        # the same seeded model unsharded on every rank (one-rank groups), for the reference
        subs = [dist.new_group([r]) for r in range(world)]
        full = TPDecoder(cfg, batch=B, device=dev, seed=7, group=subs[dist.get_rank()])
    ref = RefDecoder(full)
    toks = torch.randint(0, cfg.vocab, (B, T), generator=torch.Generator().manual_seed(4)).to(dev)
    nxt, hid = dec.prefill(toks, chunk=64, return_hidden=True)
    for t in range(T):
        xr = ref.token(toks[:, t])
    ok = True
    err = (hid.float() - xr).abs().max().item()
    scale = xr.abs().max().item()
    ok &= err <= 1e-2 * scale + 1e-2
    for step in range(4):
        cur = torch.randint(0, cfg.vocab, (B,), generator=torch.Generator().manual_seed(50 + step)).to(dev)
        nxt, hid = dec.decode_step(cur, return_hidden=True)
        xr = ref.token(cur)
        e = (hid.float() - xr).abs().max().item()
        ok &= e <= 1e-2 * xr.abs().max().item() + 1e-2
        err = max(err, e)
    print(f"rank {dist.get_rank()} world {world}: max err {err:.4g} ok={ok}", flush=True)
    import ctypes
    from qextract_infer_b200 import _lib
    code = ctypes.c_uint(0)
    assert _lib.load().qx_get_device_error(ctypes.byref(code), 1) == 0
    ok &= code.value == 0  # no bounded wait gave up
    t = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(t)
    dec.close()
    full.close()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(int(t.item() != 0))


if __name__ == "__main__":
    main()

"""Tensor-parallel sharding of the decoder checked on CPU ranks over gloo.

One small Qwen3-shaped layer (column-parallel q/k/v/gate/up, row-parallel
o/down with the LoRA partials in the same all-reduce, vocabulary-split greedy)
computed shard by shard with the numpy oracle at world sizes 2, 4 and 8, against
the unsharded oracle (rtol = atol = 1e-2).  The sharding code under test is
the decoder's own (``qextract_infer_b200.tp_shard``); see
``tests/tp_shard_worker.py``.
"""

import socket

import pytest
import torch.multiprocessing as mp

from tests import tp_shard_worker


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port):
    tp_shard_worker.run(rank, world, port)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_sharding_matches_unsharded_oracle(world, monkeypatch):
    # loopback rendezvous (the host name may not resolve) and a few threads per rank
    monkeypatch.setenv("GLOO_SOCKET_IFNAME", "lo")
    monkeypatch.setenv("OMP_NUM_THREADS", "2")
    mp.spawn(_worker, args=(world, _free_port()), nprocs=world, join=True)


def test_shard_rules_reject_bad_splits():
    import torch
    from qextract_infer_b200.tp_shard import shard_quant_linear
    qw = torch.zeros(512 // 8, 24, dtype=torch.int32)
    sc = torch.zeros(4, 24, dtype=torch.float16)
    qz = torch.zeros(4, 3, dtype=torch.int32)
    with pytest.raises(ValueError):
        shard_quant_linear(qw, sc, qz, None, None, "col", 0, 2, 128)  # 12 columns: not a multiple of 8
    with pytest.raises(ValueError):
        shard_quant_linear(qw, sc, qz, None, None, "row", 0, 8, 128)  # 64 rows: not a whole group
    out = shard_quant_linear(qw, sc, qz, None, None, "row", 1, 4, 128)
    assert out[0].shape == (16, 24) and out[1].shape == (1, 24) and out[2].shape == (1, 3)

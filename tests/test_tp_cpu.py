"""Tensor-parallel host logic on CPU ranks (gloo): sharded model == unsharded model,
INT4 shard arithmetic against the oracle, and a dead rank surfacing as an error."""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

import cases
from oracle import oracle

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch(mode: str, world: int = 2, timeout_s: float = 60, env_extra=None):
    port = free_port()
    procs = []
    for rank in range(world):
        env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                   WORLD_SIZE=str(world), LOCAL_RANK=str(rank), OMP_NUM_THREADS="1", **(env_extra or {}))
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "tp_worker.py"), mode], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
    outs = []
    for p in procs:
        try:
            out, err = p.communicate(timeout=timeout_s)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            pytest.fail(f"rank did not finish within {timeout_s} s")
        outs.append((p.returncode, out, err))
    return outs


def test_sharded_model_matches_unsharded():
    outs = launch("parity")
    for rc, out, err in outs:
        assert rc == 0, err[-2000:]
        rec = json.loads(out.strip().splitlines()[-1])
        assert rec["max_rel_err"] < 1e-5, rec
        assert rec["local_heads"] == cases.TINY_MODEL["n_heads"] // 2
        assert rec["wq_rows"] == cases.TINY_MODEL["dim"] // 2
        assert rec["w2_cols"] == 512


def test_dead_rank_is_reported_not_hung():
    outs = launch("dead_peer", timeout_s=60, env_extra={"TP_TEST_TIMEOUT": "10"})
    rc0, out0, err0 = outs[0]
    rec = json.loads(out0.strip().splitlines()[-1])
    assert rec["outcome"].startswith("error"), rec
    assert rec["seconds"] < 30


@pytest.mark.parametrize("world", [2, 4, 8])
def test_int4_shards_recombine(world):
    """Column shards concatenate and row shards sum to the unsharded INT4 product."""
    from llama.tp import shard_int4_cols, shard_int4_rows

    gen = torch.Generator().manual_seed(world)
    N, K, M = 512, 2048, 3
    w = (torch.randn(N, K, generator=gen) * 0.02).half().numpy()
    x = torch.randn(M, K, generator=gen).half().numpy()
    packed, scale, zero = (torch.from_numpy(a) for a in oracle.quantize(w, 128))
    y_full, y32_full = oracle.linear(x, packed.numpy(), scale.numpy(), zero.numpy())
    rows = [shard_int4_rows(packed, scale, zero, r, world) for r in range(world)]
    y_rows = np.concatenate([oracle.linear(x, *(t.numpy() for t in sh))[1] for sh in rows], axis=1)
    assert np.abs(y_rows - y32_full).max() <= 1e-5 * np.abs(y32_full).max()
    cols = [shard_int4_cols(packed, scale, zero, r, world, 128) for r in range(world)]
    ks = K // world
    parts = [oracle.linear(x[:, r * ks:(r + 1) * ks], *(t.numpy() for t in sh))[1] for r, sh in enumerate(cols)]
    assert np.abs(sum(parts) - y32_full).max() <= 1e-5 * np.abs(y32_full).max()


def test_shards_must_hold_whole_groups():
    from llama.tp import shard_int4_cols

    p = torch.zeros(4, 384 // 2, dtype=torch.uint8)
    s = torch.zeros(4, 3, dtype=torch.float16)
    with pytest.raises(ValueError):
        shard_int4_cols(p, s, s, 0, 2, 128)  # 384 / 2 = 192 is not a whole number of 128-groups

"""Tensor-parallel INT4 decode on 2, 4 and 8 GPUs (NCCL): the sharded tiny model matches the
unsharded one, and decode replayed from one CUDA graph (collectives inside the graph)
gives the same greedy tokens as eager decoding, as does the fused step (llama.fused) on the
shards (its vocabulary-sharded greedy step reduces per-rank argmax keys).  Runs as child
processes; each case is skipped on machines with fewer GPUs than its ranks."""
import json

import pytest
import torch

from test_tp_cpu import launch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_int4_model_matches_unsharded(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    outs = launch("gpu_parity", world=world, timeout_s=300,
                  env_extra={"NCCL_NVLS_ENABLE": "0", "TP_TEST_TIMEOUT": "120"})
    for rc, out, err in outs:
        assert rc == 0, err[-3000:]
        rec = json.loads(out.strip().splitlines()[-1])
        assert rec["prefill_rel_err"] < 1e-2, rec
        assert rec["eager_tokens_equal"] and rec["graph_tokens_equal"], rec
        assert rec["fused_graph_tokens_equal"] and rec["separate_allreduce_graph_tokens_equal"], rec


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_nvlink_allreduce_matches_nccl(world):
    """The row-parallel sum over NVLink peer memory -- li4_allreduce_add after the GEMV, and the GEMV
    that finishes the all-reduce in its own launch -- bit for bit against every rank's partial gathered
    through NCCL and summed in rank order, eager and replayed from a CUDA graph; and the greedy step over
    vocabulary shards with the keys exchanged over NVLink against torch.argmax of the gathered logits."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    outs = launch("gpu_allreduce", world=world, timeout_s=300,
                  env_extra={"NCCL_NVLS_ENABLE": "0", "TP_TEST_TIMEOUT": "120"})
    for rc, out, err in outs:
        assert rc == 0, err[-3000:]
        rec = json.loads(out.strip().splitlines()[-1])
        assert rec["bitwise_separate"] and rec["bitwise_fused"], rec
        assert rec["argmax_exchange_equal"], rec
        assert rec["device_errors"] == 0, rec

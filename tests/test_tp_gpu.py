"""Tensor-parallel INT4 decode on 2 GPUs (NCCL): the sharded tiny model matches the
unsharded one, and decode replayed from one CUDA graph (collectives inside the graph)
gives the same greedy tokens as eager decoding, as does the fused step (llama.fused) on the
shards.  Runs as child processes; skipped on
machines with fewer than 2 GPUs."""
import json

import pytest
import torch

from test_tp_cpu import launch

pytestmark = pytest.mark.gpu


def test_tp2_int4_model_matches_unsharded():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    outs = launch("gpu_parity", world=2, timeout_s=300, env_extra={"NCCL_NVLS_ENABLE": "0", "TP_TEST_TIMEOUT": "120"})
    for rc, out, err in outs:
        assert rc == 0, err[-3000:]
        rec = json.loads(out.strip().splitlines()[-1])
        assert rec["prefill_rel_err"] < 1e-2, rec
        assert rec["eager_tokens_equal"] and rec["graph_tokens_equal"], rec
        assert rec["fused_graph_tokens_equal"], rec


def test_tp2_nvlink_allreduce_matches_nccl():
    """li4_allreduce_add (one-shot over NVLink peer memory, GEMV partials written straight into the
    communication slots) against NCCL's all-reduce + residual, eager and replayed from a CUDA graph."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    outs = launch("gpu_allreduce", world=2, timeout_s=300, env_extra={"NCCL_NVLS_ENABLE": "0", "TP_TEST_TIMEOUT": "120"})
    for rc, out, err in outs:
        assert rc == 0, err[-3000:]
        rec = json.loads(out.strip().splitlines()[-1])
        assert rec["max_rel_err"] < 2e-3, rec
        assert rec["device_errors"] == 0, rec

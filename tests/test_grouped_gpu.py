"""Grouped GEMVs (li4_int4_linear_grouped): many independent INT4 GEMVs in one persistent launch,
each checked against the oracle; repeated launches and graph replays give the same bits."""
import pytest
import torch

from oracle import oracle
from test_gemv_gpu import LLAMA_SHAPES, check_close, make_problem

pytestmark = pytest.mark.gpu


def build(shapes, M, cuda_device, seed0=0):
    from llama import int4_gemv

    probs, hosts, ys = [], [], []
    for i, (_, N, K) in enumerate(shapes):
        x, p, s, z, host = make_problem(N, K, M, seed=seed0 + i, device=cuda_device)
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda_device)
        probs.append((x, p, s, z, y))
        hosts.append(host)
        ys.append(y)
    return int4_gemv.GroupedGemv(probs), hosts, ys


@pytest.mark.parametrize("M", [1, 2, 8])
def test_grouped_llama_shapes_match_oracle(M, cuda_device):
    """Every Llama-3.2-1B linear shape (lm_head included, down_proj only where M x K fits the x
    staging) in one launch, three times in a row."""
    shapes = [sh for sh in LLAMA_SHAPES if M * sh[2] * 2 <= 32768]
    grouped, hosts, ys = build(shapes, M, cuda_device)
    first = None
    for rep in range(3):
        grouped()
        torch.cuda.synchronize()
        out = [y.clone() for y in ys]
        if first is None:
            first = out
            for y, host in zip(out, hosts):
                y_ref, y32 = oracle.linear(*host)
                check_close(y, y_ref, y32, host)
        else:
            assert all(torch.equal(a, b) for a, b in zip(first, out)), "repeated launches differ"


def test_grouped_ragged_and_graph(cuda_device):
    """Odd N (partial tiles and units), different K per problem, more problems than one wave of units;
    replayed from a CUDA graph."""
    shapes = [("a", 40, 256), ("b", 1000, 1024), ("c", 129, 4096), ("d", 7, 128), ("e", 3000, 2048)] * 5
    grouped, hosts, ys = build(shapes, 3, cuda_device, seed0=100)
    grouped()
    torch.cuda.synchronize()
    ref = [y.clone() for y in ys]
    for y, host in zip(ref, hosts):
        y_ref, y32 = oracle.linear(*host)
        check_close(y, y_ref, y32, host)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        grouped()
    for y in ys:
        y.fill_(float("nan"))
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(ref, ys))

"""One rank of the CPU tensor-parallel tests (launched by tests/test_tp_cpu.py).

modes:
  parity     shard the tiny Llama over the gloo group, compare prefill and decode_step
             logits with the unsharded model on every rank; prints one JSON line
  dead_peer  rank 1 leaves right after joining; rank 0's next collective must fail
             with an error (not hang); prints one JSON line from rank 0
  gpu_parity / gpu_allreduce  the NCCL-backed GPU checks of tests/test_tp_gpu.py
"""
import datetime
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path[:0] = [REPO, os.path.join(REPO, "llama-efficient-inference_b200"), os.path.join(HERE, "golden")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def parity():
    import cases
    from llama.model import Llama, ModelArgs
    from llama.tp import shard_model

    rank, world = dist.get_rank(), dist.get_world_size()
    args = ModelArgs(**cases.TINY_MODEL)
    sd = {k: v.float() for k, v in cases.tiny_state_dict(cases.TINY_MODEL).items()}
    full = Llama(args)
    full.load_state_dict(sd)
    part = Llama(args)
    part.load_state_dict(sd)
    shard_model(part)
    prompt = cases.tiny_prompt(cases.TINY_MODEL)
    worst = 0.0
    with torch.no_grad():
        a, b = full(prompt, 0), part(prompt, 0)
        worst = max(worst, float((a - b).abs().max() / a.abs().max()))
        nxt = a[:, -1].argmax(-1, keepdim=True)
        pos = torch.tensor([prompt.shape[1]], dtype=torch.long)
        for _ in range(3):
            la, lb = full.decode_step(nxt, pos), part.decode_step(nxt, pos)
            worst = max(worst, float((la - lb).abs().max() / la.abs().max()))
            nxt = la[:, -1].argmax(-1, keepdim=True)
            pos += 1
    local_heads = part.layers[0].attention.n_local_heads
    print(json.dumps({"rank": rank, "world": world, "max_rel_err": worst, "local_heads": local_heads,
                      "wq_rows": part.layers[0].attention.wq.weight.shape[0],
                      "w2_cols": part.layers[0].feed_forward.w2.weight.shape[1]}), flush=True)


def gpu_parity():
    """NCCL ranks on GPUs: the sharded INT4 tiny model against the unsharded one, eager and graph decode."""
    import cases
    from llama import quantize
    from llama.generation import DecodeGraph, eager_tokens
    from llama.model import Llama, ModelArgs
    from llama.tp import shard_model

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", rank)
    cfg = cases.TINY_MODEL if world == 2 else cases.TP_MODEL  # 2 KV heads split 2 ways; 8 split up to 8
    args = ModelArgs(**cfg)
    sd = cases.tiny_state_dict(cfg)

    def build():
        torch.set_default_dtype(torch.float16)
        try:
            m = Llama(args)
        finally:
            torch.set_default_dtype(torch.float32)
        m.load_state_dict(sd)
        m = m.to(dev).eval()
        quantize.quantize_model(m, 128)
        return m

    quantize.set_dequant_impl("v4")
    full, part = build(), build()
    shard_model(part)
    prompt = cases.tiny_prompt(cfg).to(dev)
    steps = cases.TINY_DECODE_STEPS
    with torch.no_grad():
        a, b = full(prompt, 0), part(prompt, 0)
        prefill_err = float((a - b).abs().max() / a.abs().max())
        full.reset_cache()
        part.reset_cache()
        t_full = eager_tokens(full, prompt, steps)
        t_part = eager_tokens(part, prompt, steps)
        graph = DecodeGraph(part, prompt.shape[0])
        t_graph = graph.tokens(prompt, steps)
        torch.cuda.synchronize(dev)
        del graph
        # the fused step (llama.fused) on the shards: row-parallel partial sums all-reduced in the graph
        # (the wo / w2 GEMVs finish their own all-reduce; then with a separate all-reduce kernel)
        part.enable_fused_decode()
        fgraph = DecodeGraph(part, prompt.shape[0])
        t_fused = fgraph.tokens(prompt, steps)
        torch.cuda.synchronize(dev)
        del fgraph
        part.enable_fused_decode(fused_allreduce=False)
        sgraph = DecodeGraph(part, prompt.shape[0])
        t_sep = sgraph.tokens(prompt, steps)
        torch.cuda.synchronize(dev)
        del sgraph
    same_eager = bool(torch.equal(t_full, t_part))
    same_graph = bool(torch.equal(t_part, t_graph))
    same_fused = bool(torch.equal(t_full, t_fused))
    same_sep = bool(torch.equal(t_full, t_sep))
    print(json.dumps({"rank": rank, "world": world, "prefill_rel_err": prefill_err, "eager_tokens_equal": same_eager,
                      "graph_tokens_equal": same_graph, "fused_graph_tokens_equal": same_fused,
                      "separate_allreduce_graph_tokens_equal": same_sep}), flush=True)


def gpu_allreduce():
    """The row-parallel sum over NVLink peer memory against the same sum taken through NCCL, bit for bit:
    li4_allreduce_add after a GEMV that writes its partial into this rank's slot, and the GEMV that
    finishes the all-reduce in its own launch (LI4_EPI_ALLREDUCE_RESIDUAL); eager and replayed in a
    graph, alternating the two buffers as the decode step does, over the streaming kernel's modes
    (K-split and rows mode, with and without a split-K reduction)."""
    from llama import _native, fused
    from llama.comm import NvlinkAllReduce
    from llama.quantize import QuantizedLinear

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", rank)
    E = _native
    shapes = [(1, 2048, 2048 // world), (16, 2048, 2048 // world), (1, 2048, 8192 // world),
              (16, 2048, 8192 // world), (1, 9472, 2048), (16, 9472, 4096)]
    ar = NvlinkAllReduce(dist.group.WORLD, max_elems=max(m * n for m, n, _ in shapes), device=dev)
    bitwise_sep = bitwise_fused = True
    worst = 0.0
    with torch.no_grad():
        for M, N, K in shapes:
            gen = torch.Generator(device=dev).manual_seed(100 + rank)
            w = (torch.randn(N, K, generator=gen, device=dev) * 0.02).half()
            p, s, z = QuantizedLinear.quantize_tensor(w, 128)
            xs = [torch.randn(M, K, generator=gen, device=dev).half() for _ in range(4)]
            res = torch.randn(M, N, generator=torch.Generator(device=dev).manual_seed(7), device=dev).half()
            sep = [torch.empty(M, N, dtype=torch.float16, device=dev) for _ in range(4)]
            fus = [torch.empty(M, N, dtype=torch.float16, device=dev) for _ in range(4)]

            def run():
                for i, x in enumerate(xs):
                    fused.int4_linear_fused(x, p, s, z, None, E.Fusion(epilogue=E.LI4_EPI_STORE),
                                            y_ptr=ar.slot_ptr(i % 2), y_stride=N)
                    ar.all_reduce_add(i % 2, res, sep[i])
                for i, x in enumerate(xs):
                    fused.int4_linear_fused(x, p, s, z, fus[i], ar.push_fusion(i % 2, res))

            refs = []  # every rank's partial gathered, summed in fp32 in rank order, + residual
            for x in xs:
                part = torch.empty(M, N, dtype=torch.float16, device=dev)
                fused.int4_linear_fused(x, p, s, z, part, E.Fusion(epilogue=E.LI4_EPI_STORE))
                parts = [torch.empty_like(part) for _ in range(world)]
                dist.all_gather(parts, part)
                acc = torch.zeros(M, N, dtype=torch.float32, device=dev)
                for t in parts:
                    acc += t.float()
                refs.append((res.float() + acc.half().float()).half())

            def check():
                nonlocal bitwise_sep, bitwise_fused, worst
                for a, b, r in zip(sep, fus, refs):
                    bitwise_sep &= bool(torch.equal(a, r))
                    bitwise_fused &= bool(torch.equal(b, r))
                    worst = max(worst, float((b.float() - r.float()).abs().max() / r.float().abs().max()))

            for _ in range(3):
                run()
            torch.cuda.synchronize(dev)
            check()
            g = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                run()
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(g):
                run()
            for o in sep + fus:
                o.zero_()
            for _ in range(5):
                g.replay()
            torch.cuda.synchronize(dev)
            check()
            del g
        # the greedy step over vocabulary shards (li4_argmax_rows_allreduce) against torch.argmax of the
        # gathered logits: random rows, a row whose maximum every shard shares (the first index wins)
        # and fp16 logits; eager calls and graph replays
        rows, shard = 16, 1000
        lg = torch.Generator(device=dev).manual_seed(55 + rank)
        keys_ok = True
        for dtype in (torch.float32, torch.float16):
            for trial in range(3):
                logits = torch.randn(rows, shard, generator=lg, device=dev).to(dtype)
                logits[3, 17] = 50.0  # the same maximum in every shard: rank 0's column 17 wins
                full = [torch.empty_like(logits) for _ in range(world)]
                dist.all_gather(full, logits)
                want = torch.cat(full, 1).float().argmax(-1)
                out = torch.full((rows, 1), -1, dtype=torch.long, device=dev)
                ar.argmax_allreduce(logits, rank * shard, out)
                torch.cuda.synchronize(dev)
                keys_ok &= bool(torch.equal(out.view(-1), want))
            g = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                ar.argmax_allreduce(logits, rank * shard, out)
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(g):
                ar.argmax_allreduce(logits, rank * shard, out)
            for _ in range(3):
                out.fill_(-1)
                g.replay()
                torch.cuda.synchronize(dev)
                keys_ok &= bool(torch.equal(out.view(-1), want))
            del g
    errors = _native.device_errors()
    dist.barrier()
    ar.close()
    print(json.dumps({"rank": rank, "world": world, "bitwise_separate": bitwise_sep, "bitwise_fused": bitwise_fused,
                      "argmax_exchange_equal": keys_ok, "max_rel_err": worst, "device_errors": errors}), flush=True)


def dead_peer():
    rank = dist.get_rank()
    if rank == 1:
        os._exit(0)  # leaves between steps, with nothing in flight
    time.sleep(1.0)
    t0 = time.time()
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
        outcome = "no error"
    except Exception as e:  # noqa: BLE001 -- the failure is the expected outcome
        outcome = f"error: {type(e).__name__}"
    print(json.dumps({"rank": rank, "outcome": outcome, "seconds": round(time.time() - t0, 2)}), flush=True)


if __name__ == "__main__":
    mode = sys.argv[1]
    timeout = datetime.timedelta(seconds=float(os.environ.get("TP_TEST_TIMEOUT", "60")))
    if mode in ("gpu_parity", "gpu_allreduce"):
        torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
        dist.init_process_group("nccl", timeout=timeout,
                                device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    else:
        dist.init_process_group("gloo", timeout=timeout)
    {"parity": parity, "dead_peer": dead_peer, "gpu_parity": gpu_parity, "gpu_allreduce": gpu_allreduce}[mode]()
    if mode in ("parity", "gpu_parity", "gpu_allreduce"):
        dist.barrier()
        dist.destroy_process_group()
    os._exit(0)

"""Generation loop with CUDA-graph decode (the reference's llama/generation.py:5-93 plus
the graph capture its bench.py:103-151 does per position).

DecodeGraph captures ONE graph of the per-token step -- embedding, 16 blocks with the
INT4 GEMV kernels, lm_head, greedy argmax, position increment -- and replays it for
every position: the position lives in a device tensor (Llama.decode_step), so
nothing position-dependent is baked into the graph.  Replays chain on the GPU: each
reads the token buffer, writes the argmax back into it and advances the position.
"""
from __future__ import annotations

import torch
from torch import nn


class DecodeGraph:
    """Greedy decode steps replayed from one CUDA graph.

    tok [bs, 1] int64 and pos [1] int64 are static device buffers; replay() runs
    one step at position pos and leaves the next token in tok, pos + 1 in pos.
    With capture_logits, the step's fp32 logits stay readable in .logits.
    """

    @torch.no_grad()
    def __init__(self, model: nn.Module, bs: int, warmup: int = 2):
        self.model, self.bs = model, bs
        dev = next(model.parameters()).device if any(True for _ in model.parameters()) else \
            next(model.buffers()).device
        self.device = dev
        self.tok = torch.zeros(bs, 1, dtype=torch.long, device=dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        saved = self.pos.clone()
        with torch.cuda.stream(side):
            for _ in range(warmup):  # sizes every buffer and workspace before capture
                self._step()
            self.pos.copy_(saved)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = self._step()
        torch.cuda.synchronize(dev)

    def _step(self):
        fused = getattr(self.model, "_fused", None)
        if fused is not None:  # fused step: the greedy argmax and pos += 1 run on the GPU kernels
            return fused.decode_step(self.tok, self.pos, next_tokens=self.tok, advance_pos=True)
        logits = self.model.decode_step(self.tok, self.pos)
        self.tok.copy_(logits[:, -1].argmax(-1, keepdim=True))
        self.pos.add_(1)
        return logits

    @torch.no_grad()
    def start(self, tokens: torch.Tensor, start_pos: int = 0):
        """Eager prefill of tokens [bs, s] at start_pos; leaves the first greedy token in tok."""
        logits = self.model(tokens, start_pos)
        self.tok.copy_(logits[:, -1].argmax(-1, keepdim=True))
        self.pos.fill_(start_pos + tokens.shape[1])
        return logits

    def replay(self):
        self.graph.replay()

    @torch.no_grad()
    def tokens(self, tokens: torch.Tensor, n_steps: int) -> torch.Tensor:
        """Prefill, then n_steps replays; the greedy tokens [bs, 1 + n_steps]."""
        self.start(tokens)
        out = [self.tok.clone()]
        for _ in range(n_steps):
            self.replay()
            out.append(self.tok.clone())
        return torch.cat(out, 1)


@torch.no_grad()
def eager_tokens(model: nn.Module, tokens: torch.Tensor, n_steps: int) -> torch.Tensor:
    """Greedy tokens from the eager reference-style loop (the reference's bench.py:154-161)."""
    _, input_len = tokens.shape
    nxt = model(tokens, 0)[:, -1].argmax(-1, keepdim=True)
    out = [nxt]
    for i in range(n_steps):
        nxt = model(nxt, input_len + i)[:, -1].argmax(-1, keepdim=True)
        out.append(nxt)
    return torch.cat(out, 1)


class Generation(nn.Module):
    def generate(self, tokenizer, prompts, max_gen_len, temperature, top_p, kv_caching, device, cuda_graph=False):
        """The reference's generate (llama/generation.py:6-82).  cuda_graph=True replays the
        decode steps from one captured graph (greedy: temperature must be 0)."""
        prompt_tokens = [tokenizer.encode(x, bos=True, eos=False) for x in prompts]
        bsz = len(prompt_tokens)
        min_prompt_len = min(len(t) for t in prompt_tokens)
        max_prompt_len = max(len(t) for t in prompt_tokens)
        total_len = max_gen_len + max_prompt_len
        tokens = torch.full((bsz, total_len), tokenizer.pad_id, dtype=torch.long, device=device)
        for k, t in enumerate(prompt_tokens):
            tokens[k, : len(t)] = torch.tensor(t, dtype=torch.long, device=device)
        eos_reached = torch.tensor([False] * bsz, device=device)
        input_text_mask = tokens != tokenizer.pad_id
        graph = None
        if cuda_graph:
            if not kv_caching or temperature > 0:
                raise ValueError("cuda_graph decode needs kv_caching=True and greedy sampling (temperature 0)")
            graph = DecodeGraph(self, bsz)
        prev_pos = 0
        for cur_pos in range(min_prompt_len, total_len):
            with torch.no_grad():
                if not kv_caching:
                    # decoding without the cache: reprocess the whole prefix each step
                    logits = self(tokens[:, :cur_pos], 0)
                elif graph is not None and prev_pos > 0:
                    graph.tok.copy_(tokens[:, prev_pos:cur_pos])
                    graph.pos.fill_(prev_pos)
                    graph.replay()
                    logits = graph.logits
                else:
                    logits = self(tokens[:, prev_pos:cur_pos], prev_pos)
            if temperature > 0:
                probs = torch.softmax(logits[:, -1] / temperature, dim=-1)
                next_token = sample_top_p(probs, top_p)
            else:
                next_token = torch.argmax(logits[:, -1], dim=-1)
            next_token = next_token.reshape(-1)
            next_token = torch.where(input_text_mask[:, cur_pos], tokens[:, cur_pos], next_token)
            tokens[:, cur_pos] = next_token
            eos_reached |= (~input_text_mask[:, cur_pos]) & (next_token == tokenizer.eos_id)
            if kv_caching:
                prev_pos = cur_pos
            if all(eos_reached):
                break
        out_tokens = []
        for i, toks in enumerate(tokens.tolist()):
            start = len(prompt_tokens[i])
            toks = toks[start: len(prompt_tokens[i]) + max_gen_len]
            if tokenizer.eos_id in toks:
                toks = toks[: toks.index(tokenizer.eos_id)]
            out_tokens.append(toks)
        return [{"generation": tokenizer.decode(t)} for t in out_tokens]


def sample_top_p(probs, p):
    """Nucleus sampling (llama/generation.py:85-93)."""
    probs_sort, probs_idx = torch.sort(probs, dim=-1, descending=True)
    probs_sum = torch.cumsum(probs_sort, dim=-1)
    mask = probs_sum - probs_sort > p
    probs_sort[mask] = 0.0
    probs_sort.div_(probs_sort.sum(dim=-1, keepdim=True))
    next_token = torch.multinomial(probs_sort, num_samples=1)
    return torch.gather(probs_idx, -1, next_token)

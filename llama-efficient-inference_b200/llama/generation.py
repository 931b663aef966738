"""Generation loop with CUDA-graph decode: the reference's interface (llama/generation.py:5-93)
around one reusable decode graph (its bench.py:103-151 captures one graph per position).

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
    """Text generation over the model's forward / decode step (the reference's interface,
    llama/generation.py:5-82).

    A batch of prompts is laid out in one token buffer, padded to the longest prompt plus
    max_gen_len.  Decoding starts at the shortest prompt's length: each step produces the next
    token of every sequence, but sequences still inside their prompt keep the prompt token
    (teacher forcing), and a sequence stops contributing once it emits eos.  With the KV cache
    each step feeds only the positions since the previous step; without it, the whole prefix.
    cuda_graph=True (greedy only) runs the first step eagerly and every later one by replaying a
    DecodeGraph, whose own greedy token is used directly."""

    def generate(self, tokenizer, prompts, max_gen_len, temperature, top_p, kv_caching, device, cuda_graph=False):
        encoded = [tokenizer.encode(text, bos=True, eos=False) for text in prompts]
        lengths = [len(t) for t in encoded]
        first, total = min(lengths), max(lengths) + max_gen_len
        buf = torch.full((len(encoded), total), tokenizer.pad_id, dtype=torch.long, device=device)
        for row, toks in enumerate(encoded):
            buf[row, :len(toks)] = torch.tensor(toks, dtype=torch.long, device=device)
        in_prompt = buf != tokenizer.pad_id
        finished = torch.zeros(len(encoded), dtype=torch.bool, device=device)
        if cuda_graph and (not kv_caching or temperature > 0):
            raise ValueError("cuda_graph decode needs kv_caching=True and greedy sampling (temperature 0)")
        graph = DecodeGraph(self, len(encoded)) if cuda_graph else None
        fed = 0  # positions already in the KV cache
        for pos in range(first, total):
            with torch.no_grad():
                if graph is not None and fed > 0:  # one position since the last step: replay the graph
                    graph.tok.copy_(buf[:, fed:pos])
                    graph.pos.fill_(fed)
                    graph.replay()
                    choice = graph.tok.view(-1).clone()
                else:
                    logits = self(buf[:, fed:pos], fed) if kv_caching else self(buf[:, :pos], 0)
                    last = logits[:, -1]
                    if temperature > 0:
                        choice = sample_top_p(torch.softmax(last / temperature, dim=-1), top_p).view(-1)
                    else:
                        choice = last.argmax(dim=-1)
            choice = torch.where(in_prompt[:, pos], buf[:, pos], choice)
            buf[:, pos] = choice
            finished |= ~in_prompt[:, pos] & (choice == tokenizer.eos_id)
            if kv_caching:
                fed = pos
            if bool(finished.all()):
                break
        results = []
        for row, n in enumerate(lengths):
            gen = buf[row, n:n + max_gen_len].tolist()
            if tokenizer.eos_id in gen:
                gen = gen[:gen.index(tokenizer.eos_id)]
            results.append({"generation": tokenizer.decode(gen)})
        return results


def sample_top_p(probs, p):
    """Nucleus sampling (llama/generation.py:85-93): draw from the smallest set of most likely tokens
    whose probability mass reaches p, renormalised; returns the drawn token ids [..., 1]."""
    ranked, order = probs.sort(dim=-1, descending=True)
    mass_above = ranked.cumsum(dim=-1) - ranked  # probability of the tokens ranked before each one
    kept = ranked.masked_fill(mass_above > p, 0.0)
    drawn = torch.multinomial(kept / kept.sum(dim=-1, keepdim=True), num_samples=1)
    return order.gather(-1, drawn)

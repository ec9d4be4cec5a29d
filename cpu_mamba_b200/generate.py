"""Autoregressive generation on the GPU around forward_step.

The reference's README (README.md:75-86) sketches the loop: prefill the prompt
once with forward_with_final_state, then forward_step token by token -- "sample,
append, repeat" -- with the sampling left to the caller.  Here the whole loop
stays on the device: a sampler maps each step's output y (B, d_model) to the
next step's input and a token id in device ops only, so ``steps_per_graph``
consecutive steps (model step + sampling) are captured as ONE CUDA graph and
replayed; the host neither waits for nor reads a token until the end.

Any model with ``forward_with_final_state`` / ``forward_step`` works: a
CPUMamba, a MambaStack, or a ChannelShardedMamba (whose graph then holds its
all-reduces).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F


class TiedEmbeddingSampler:
    """Token choice through an LM head tied to the input embedding (the
    Mamba language-model layout): logits = RMSNorm(y) E^T (the norm skipped
    when ``norm_weight`` is None), token = argmax (``temperature`` 0) or a
    sample of softmax(logits / temperature), optionally over the ``top_k``
    largest logits only (Gumbel-max with the device's default generator, so
    it can be captured in a graph).  Returns (E[token], token)."""

    def __init__(self, embedding: torch.Tensor, temperature: float = 0.0,
                 top_k: Optional[int] = None, norm_weight: Optional[torch.Tensor] = None,
                 eps: float = 1e-5):
        if embedding.dim() != 2:
            raise ValueError("embedding must be (vocab, d_model)")
        if temperature < 0:
            raise ValueError("temperature must be >= 0")
        self.E = embedding
        self.temperature = float(temperature)
        self.top_k = top_k
        self.norm_weight = norm_weight
        self.eps = eps

    def logits(self, y: torch.Tensor) -> torch.Tensor:
        h = y
        if self.norm_weight is not None:
            h = F.rms_norm(y.float(), (y.shape[-1],), self.norm_weight.float(), self.eps)
        return h.float() @ self.E.float().t()

    def __call__(self, y: torch.Tensor) -> tuple:
        z = self.logits(y)
        if self.temperature == 0.0:
            tok = z.argmax(dim=-1)
        else:
            z = z / self.temperature
            u = torch.rand_like(z).clamp_(min=1e-20, max=1.0 - 1e-7)
            g = z - torch.log(-torch.log(u))
            if self.top_k is not None and self.top_k < z.shape[-1]:
                kth = torch.topk(z, self.top_k, dim=-1).values[:, -1:]
                g = torch.where(z >= kth, g, torch.full_like(g, float("-inf")))
            tok = g.argmax(dim=-1)
        return self.E[tok].to(y.dtype), tok


class DecodeLoop:
    """``steps_per_graph`` decode steps (model step + sampler) captured as one
    CUDA graph over a fixed state.  ``run(n)`` advances the state by n tokens
    and returns their ids (B, n): whole graph replays, then eager steps for
    the remainder (the same kernels, so the same bits).  The next input lives
    in ``self.x``; ``prefill`` sets it from a prompt."""

    def __init__(self, model, sampler, state, x0: torch.Tensor, steps_per_graph: int = 16):
        if steps_per_graph < 1:
            raise ValueError("steps_per_graph must be >= 1")
        self.model, self.sampler, self.state = model, sampler, state
        self.K = int(steps_per_graph)
        self.x = x0.detach().clone().contiguous()
        self.tokens = torch.empty(self.K, x0.shape[0], dtype=torch.long, device=x0.device)
        dev = self.x.device
        # warm-up on copies (library and sampler set-up outside the capture)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.no_grad():
            self._steps(self.x.clone(), _clone_state(state), torch.empty_like(self.tokens), 1)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph):
            x_last = self._steps(self.x, self.state, self.tokens, self.K)
            self.x.copy_(x_last)

    def _steps(self, x, state, tokens, n):
        for k in range(n):
            y, _ = self.model.forward_step(x, state)
            x, tok = self.sampler(y)
            tokens[k].copy_(tok)
        return x

    @torch.no_grad()
    def run(self, n: int) -> torch.Tensor:
        out = []
        for _ in range(n // self.K):
            self.graph.replay()
            out.append(self.tokens.t().clone())
        r = n % self.K
        if r:
            tok = torch.empty(r, self.x.shape[0], dtype=torch.long, device=self.x.device)
            self.x.copy_(self._steps(self.x.clone(), self.state, tok, r))
            out.append(tok.t())
        if not out:
            return torch.empty(self.x.shape[0], 0, dtype=torch.long, device=self.x.device)
        return torch.cat(out, dim=1)


def _clone_state(state):
    if isinstance(state, dict):
        return {k: v.clone() for k, v in state.items()}
    return [_clone_state(s) for s in state]


@torch.no_grad()
def generate(model, sampler, prompt: torch.Tensor, max_new_tokens: int,
             steps_per_graph: int = 16) -> tuple:
    """Prefill ``prompt`` (B, T, d_model) with forward_with_final_state, pick
    the first token from its last position, then decode ``max_new_tokens`` - 1
    more on the GPU.  Returns (tokens (B, max_new_tokens), final state)."""
    if max_new_tokens < 1:
        raise ValueError("max_new_tokens must be >= 1")
    y, state = model.forward_with_final_state(prompt)
    x, tok0 = sampler(y[:, -1])
    rest = max_new_tokens - 1
    if rest == 0:
        return tok0[:, None], state
    loop = DecodeLoop(model, sampler, state, x, min(steps_per_graph, rest))
    return torch.cat([tok0[:, None], loop.run(rest)], dim=1), state

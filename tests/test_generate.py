"""Decode of a residual stack and the on-GPU generation loop.

CPU: the tied-embedding sampler's token choice (greedy = argmax of the logits,
top-k sampling stays inside the top k).  GPU: MambaStack.forward_with_final_state
leaves the same output as forward() and per-layer states from which
forward_step continues the sequence (against the oracle's stack over the whole
sequence, fp32 2e-5 max abs / bf16 mean rel err 2e-2); the graph-captured
DecodeLoop yields the same tokens as the same steps run eagerly."""
import pytest
import torch

import oracle
from cpu_mamba_b200 import CPUMamba, MambaStack
from cpu_mamba_b200.generate import DecodeLoop, TiedEmbeddingSampler, generate

DEV = "cuda:0"


def test_greedy_sampler_is_argmax_of_tied_logits():
    g = torch.Generator().manual_seed(0)
    E = torch.randn(50, 16, generator=g)
    y = torch.randn(4, 16, generator=g)
    x, tok = TiedEmbeddingSampler(E)(y)
    assert torch.equal(tok, (y @ E.t()).argmax(-1))
    assert torch.equal(x, E[tok])
    nw = torch.rand(16, generator=g) + 0.5
    _, tok = TiedEmbeddingSampler(E, norm_weight=nw)(y)
    ref = torch.nn.functional.rms_norm(y, (16,), nw, 1e-5) @ E.t()
    assert torch.equal(tok, ref.argmax(-1))


def test_top_k_sampling_stays_in_the_top_k():
    torch.manual_seed(1)
    E = torch.randn(40, 8)
    y = torch.randn(64, 8)
    s = TiedEmbeddingSampler(E, temperature=1.5, top_k=3)
    top = torch.topk(y @ E.t(), 3, dim=-1).indices
    for _ in range(5):
        _, tok = s(y)
        assert bool((top == tok[:, None]).any(-1).all())
    with pytest.raises(ValueError):
        TiedEmbeddingSampler(E, temperature=-1)


def _stack(dtype=torch.float32, n=3, dm=64, S=16, seed=2):
    s = MambaStack(n, dm, d_state=S)
    layers = []
    for i, layer in enumerate(s.layers):
        p = oracle.make_block_params(dm, S, seed=seed + i)
        layer.mixer.load_state_dict(p)
        g = torch.rand(dm, generator=torch.Generator().manual_seed(40 + i)) + 0.5
        with torch.no_grad():
            layer.norm.weight.copy_(g)
        layers.append((p, g))
    return s.to(DEV, dtype), layers


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_stack_prefill_then_steps(dtype):
    B, T, extra, dm = 3, 37, 6, 64
    s, layers = _stack(dtype)
    x = torch.randn(B, T + extra, dm, generator=torch.Generator().manual_seed(9))
    ref = oracle.stack_forward(layers, x, eps=s.eps)           # the whole sequence
    xd = x.to(DEV, dtype)
    with torch.no_grad():
        y, states = s.forward_with_final_state(xd[:, :T])
        assert torch.equal(y, s(xd[:, :T]))
        ys = [s.forward_step(xd[:, t], states)[0] for t in range(T, T + extra)]
    got = torch.cat([y.float().cpu(), torch.stack(ys, 1).float().cpu()], dim=1)
    if dtype == torch.float32:
        assert (got - ref).abs().max().item() <= 2e-5
    else:
        rel = ((got - ref).abs() / (ref.abs().clamp(min=1e-3) + 1e-6)).mean().item()
        assert rel <= 2e-2


class _FirstFeaturesSampler:
    """A sampler without library GEMMs (so the graph and eager runs use the
    same kernels): token = argmax of the first V features, input = E[token]."""

    def __init__(self, E):
        self.E = E

    def __call__(self, y):
        tok = y[:, : self.E.shape[0]].float().argmax(-1)
        return self.E[tok].to(y.dtype), tok


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["block", "stack"])
def test_graph_decode_loop_matches_eager_steps(kind):
    B, T, dm, V = 4, 20, 64, 48
    if kind == "block":
        m = CPUMamba(dm, 16)
        m.load_state_dict(oracle.make_block_params(dm, 16, seed=5))
        m = m.to(DEV)
    else:
        m, _ = _stack()
    E = torch.randn(V, dm, generator=torch.Generator().manual_seed(6)).to(DEV)
    sampler = _FirstFeaturesSampler(E)
    prompt = torch.randn(B, T, dm, generator=torch.Generator().manual_seed(7)).to(DEV)
    with torch.no_grad():
        toks, _ = generate(m, sampler, prompt, 1 + 8 * 2 + 3, steps_per_graph=8)
        # the same loop, eagerly
        y, st = m.forward_with_final_state(prompt)
        x, tok = sampler(y[:, -1])
        ref = [tok]
        for _ in range(8 * 2 + 3):
            y, st = m.forward_step(x, st)
            x, tok = sampler(y)
            ref.append(tok)
    assert torch.equal(toks, torch.stack(ref, 1))


@pytest.mark.gpu
def test_generate_with_tied_head_runs_in_a_graph():
    m, _ = _stack(n=2)
    E = torch.randn(100, 64, generator=torch.Generator().manual_seed(8)).to(DEV)
    s = TiedEmbeddingSampler(E, temperature=0.8, top_k=10,
                             norm_weight=torch.ones(64, device=DEV))
    prompt = E[torch.randint(0, 100, (2, 12), generator=torch.Generator().manual_seed(9))
               .to(DEV)]
    toks, states = generate(m, s, prompt, 33, steps_per_graph=16)
    assert toks.shape == (2, 33) and toks.dtype == torch.long
    assert int(toks.min()) >= 0 and int(toks.max()) < 100
    assert len(states) == 2 and torch.isfinite(states[0]["h"]).all()
    with pytest.raises(ValueError):
        DecodeLoop(m, s, states, E[:2], steps_per_graph=0)

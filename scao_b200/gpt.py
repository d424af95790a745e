"""GPT-2-shaped language model and one data-parallel training step with the
SCAO optimizer -- the caller of the optimizer step in benchmark configuration C3
(GPT-2-medium: 24 layers, d = 1024, 16 heads, d_ff = 4096, vocab 50257,
8 x 1024 tokens, bf16 autocast, fp32 optimizer state).

The architecture follows the reference's benchmark model
(scao/benchmarks/gpt_scale_benchmark.py:79-170): fused bias-free QKV and
output projections, bias-free GELU MLP, pre-LayerNorm blocks, learned
positions, LM head tied to the token embedding, N(0, 0.02^2) init.

``train_step`` runs forward / backward under bf16 autocast, then the SCAO step:
on one GPU ``opt.step()``; across ranks the owner-compute ``ShardedSCAO``
(gradient reduce-scatter with averaging, owned step, parameter all-gather),
which is the data-parallel step -- every rank ends with identical weights.
After ``sharded.attach_grad_hooks()`` the gradient reduce-scatter of each
bucket starts during backward instead of after it.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class GPTConfig:
    n_layer: int = 24
    d_model: int = 1024
    n_head: int = 16
    d_ff: int = 4096
    vocab: int = 50257
    seq_len: int = 1024


GPT2_MEDIUM = GPTConfig()


class _Attention(nn.Module):
    def __init__(self, c: GPTConfig):
        super().__init__()
        self.n_head = c.n_head
        self.qkv = nn.Linear(c.d_model, 3 * c.d_model, bias=False)
        self.proj = nn.Linear(c.d_model, c.d_model, bias=False)

    def forward(self, x):
        B, T, C = x.shape
        q, k, v = self.qkv(x).split(C, dim=2)
        heads = lambda t: t.view(B, T, self.n_head, C // self.n_head).transpose(1, 2)
        y = F.scaled_dot_product_attention(heads(q), heads(k), heads(v), is_causal=True)
        return self.proj(y.transpose(1, 2).reshape(B, T, C))


class _Block(nn.Module):
    def __init__(self, c: GPTConfig):
        super().__init__()
        self.ln1 = nn.LayerNorm(c.d_model)
        self.attn = _Attention(c)
        self.ln2 = nn.LayerNorm(c.d_model)
        self.fc = nn.Linear(c.d_model, c.d_ff, bias=False)
        self.out = nn.Linear(c.d_ff, c.d_model, bias=False)

    def forward(self, x):
        x = x + self.attn(self.ln1(x))
        return x + self.out(F.gelu(self.fc(self.ln2(x))))


class GPT(nn.Module):
    def __init__(self, c: GPTConfig = GPT2_MEDIUM, seed: int = 0):
        super().__init__()
        self.c = c
        self.tok = nn.Embedding(c.vocab, c.d_model)
        self.pos = nn.Embedding(c.seq_len, c.d_model)
        self.blocks = nn.ModuleList([_Block(c) for _ in range(c.n_layer)])
        self.ln_f = nn.LayerNorm(c.d_model)
        self.head = nn.Linear(c.d_model, c.vocab, bias=False)
        self.head.weight = self.tok.weight
        g = torch.Generator().manual_seed(seed)
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)) and m is not self.head:
                with torch.no_grad():
                    m.weight.copy_(torch.randn(m.weight.shape, generator=g) * 0.02)

    def forward(self, idx):
        T = idx.shape[1]
        x = self.tok(idx) + self.pos(torch.arange(T, device=idx.device))
        for b in self.blocks:
            x = b(x)
        return self.head(self.ln_f(x))


def token_batch(c: GPTConfig, batch: int, seed: int, device):
    """``batch`` sequences of ``seq_len + 1`` tokens uniform over the vocabulary."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    t = torch.randint(0, c.vocab, (batch, c.seq_len + 1), generator=g)
    return t.to(device)


def loss_fn(model, tokens):
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits = model(tokens[:, :-1])
    return F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]),
                           tokens[:, 1:].reshape(-1))


def train_step(model, opt, tokens, sharded=None):
    """Forward + backward (bf16 autocast) + SCAO step; returns the loss."""
    loss = loss_fn(model, tokens)
    loss.backward()
    if sharded is not None:
        sharded.flat_grad_from_params()
        sharded.step()
    else:
        opt.step()
    model.zero_grad(set_to_none=True)
    return loss.detach()

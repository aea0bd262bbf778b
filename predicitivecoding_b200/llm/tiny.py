"""Single-block causal transformer LM and plain SGD, the autograd engine's smallest client.

Reference: PredictiveCoding.LLM/Autograd/TinyTransformerLM.cs:12-121 (one pre-LN block, attention
scale 1/sqrt(dim) over the full width, GELU FFN with biases, untied output [dim, vocab], weights
N(0, 0.02^2); ``Sgd.Step`` p -= lr * grad).
"""
from __future__ import annotations

import math
from typing import List, Sequence

import torch
import torch.nn.functional as F


class TinyTransformerLM:
    def __init__(self, vocab: int, dim: int, ff: int, seed: int = 0, eps: float = 1e-5, dropout: float = 0.0):
        g = torch.Generator().manual_seed(seed)

        def randn(r, c):
            return (torch.randn(r, c, generator=g) * 0.02).requires_grad_()

        self.vocab, self.dim, self.eps, self.dropout = vocab, dim, eps, dropout
        self.attn_scale = 1.0 / math.sqrt(dim)
        self.wemb = randn(vocab, dim)
        self.wq, self.wk, self.wv, self.wo = randn(dim, dim), randn(dim, dim), randn(dim, dim), randn(dim, dim)
        self.ln1_g, self.ln1_b = torch.ones(dim, requires_grad=True), torch.zeros(dim, requires_grad=True)
        self.ln2_g, self.ln2_b = torch.ones(dim, requires_grad=True), torch.zeros(dim, requires_grad=True)
        self.w1, self.b1 = randn(dim, ff), torch.zeros(ff, requires_grad=True)
        self.w2, self.b2 = randn(ff, dim), torch.zeros(dim, requires_grad=True)
        self.wout = randn(dim, vocab)

    def parameters(self) -> List[torch.Tensor]:
        return [self.wemb, self.wq, self.wk, self.wv, self.wo, self.ln1_g, self.ln1_b, self.ln2_g, self.ln2_b,
                self.w1, self.b1, self.w2, self.b2, self.wout]

    def forward(self, tokens: Sequence[int], training: bool = False) -> torch.Tensor:
        t = torch.as_tensor(tokens, dtype=torch.long)
        S = t.numel()
        x = self.wemb[t]
        h1 = F.layer_norm(x, (self.dim,), self.ln1_g, self.ln1_b, self.eps)
        q, k, v = h1 @ self.wq, h1 @ self.wk, h1 @ self.wv
        s = (q @ k.T) * self.attn_scale
        s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool), 1), float("-inf"))
        a = torch.softmax(s, -1) @ v
        x = x + F.dropout(a @ self.wo, self.dropout, training)
        h2 = F.layer_norm(x, (self.dim,), self.ln2_g, self.ln2_b, self.eps)
        f = F.gelu(h2 @ self.w1 + self.b1, approximate="tanh") @ self.w2 + self.b2
        x = x + F.dropout(f, self.dropout, training)
        return x @ self.wout

    def loss(self, tokens, targets, training: bool = False) -> torch.Tensor:
        return F.cross_entropy(self.forward(tokens, training), torch.as_tensor(targets, dtype=torch.long))


def sgd_step(parameters, lr: float) -> None:
    with torch.no_grad():
        for p in parameters:
            if p.grad is not None:
                p -= lr * p.grad

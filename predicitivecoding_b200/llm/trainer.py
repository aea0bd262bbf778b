"""Mini-batch training steps for the autograd decoder.

Reference: PredictiveCoding.LLM/Training/Trainer.cs:13-209.  ``step`` zeroes gradients,
runs forward/backward per window, averages the summed gradients over the batch,
clips and applies Adam.  ``step_parallel`` splits the batch into balanced contiguous
shards processed by worker replicas (threads here; one rank per GPU belongs to the
fused trainer) and merges the shard gradients in fixed worker order, so the result
is reproducible run to run.
"""
from __future__ import annotations

import threading
from typing import Callable, List, Sequence, Tuple

import torch

from ..optim.adam import Adam, clip_global_norm

LossFn = Callable[[torch.Tensor, torch.Tensor, bool], torch.Tensor]


def _window_tensors(w, device):
    t, y = w
    return (torch.as_tensor(t, dtype=torch.long, device=device), torch.as_tensor(y, dtype=torch.long, device=device))


def step(params: Sequence[torch.Tensor], batch: Sequence[Tuple], loss_fn: LossFn, optimizer: Adam, lr: float,
         clip_norm: float = None, training: bool = True) -> float:
    device = params[0].device
    acc = [torch.zeros_like(p) for p in params]
    total = 0.0
    for w in batch:
        for p in params:
            p.grad = None
        t, y = _window_tensors(w, device)
        loss = loss_fn(t, y, training)
        loss.backward()
        total += float(loss.detach())
        for a, p in zip(acc, params):
            if p.grad is not None:
                a.add_(p.grad)
    b = max(1, len(batch))
    for a, p in zip(acc, params):
        p.grad = a / b
    if clip_norm is not None:
        clip_global_norm(params, clip_norm)
    optimizer.step(params, lr)
    return total / b


def shard_bounds(count: int, workers: int) -> List[int]:
    base, extra = divmod(count, workers)
    bounds, pos = [0], 0
    for w in range(workers):
        pos += base + (1 if w < extra else 0)
        bounds.append(pos)
    return bounds


def step_parallel(replicas: Sequence[Sequence[torch.Tensor]], loss_fns: Sequence[LossFn], batch: Sequence[Tuple],
                  optimizer: Adam, lr: float, clip_norm: float = None, training: bool = True) -> float:
    workers = len(replicas)
    if workers == 0:
        raise ValueError("Need at least one replica.")
    if len(loss_fns) != workers:
        raise ValueError("One loss function per replica is required.")
    primary = replicas[0]
    with torch.no_grad():
        for w in range(1, workers):
            for a, b in zip(primary, replicas[w]):
                b.copy_(a)
    bounds = shard_bounds(len(batch), workers)
    grads: List[List[torch.Tensor]] = [None] * workers
    losses = [0.0] * workers

    def run(w):
        ps = replicas[w]
        acc = [torch.zeros_like(p) for p in ps]
        s = 0.0
        for e in range(bounds[w], bounds[w + 1]):
            for p in ps:
                p.grad = None
            t, y = _window_tensors(batch[e], ps[0].device)
            loss = loss_fns[w](t, y, training)
            loss.backward()
            s += float(loss.detach())
            for a, p in zip(acc, ps):
                if p.grad is not None:
                    a.add_(p.grad)
        grads[w], losses[w] = acc, s

    if workers == 1:
        run(0)
    else:
        threads = [threading.Thread(target=run, args=(w,)) for w in range(workers)]
        for th in threads:
            th.start()
        for th in threads:
            th.join()
    b = max(1, len(batch))
    for k, p in enumerate(primary):
        g = torch.zeros_like(p)
        for w in range(workers):         # fixed merge order
            g.add_(grads[w][k])
        p.grad = g / b
    if clip_norm is not None:
        clip_global_norm(primary, clip_norm)
    optimizer.step(primary, lr)
    return sum(losses) / b

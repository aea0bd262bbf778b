"""Byte-LM quality parity: the fused device trainer and the plain PyTorch baseline trained from the same
initial weights on the same batches, then scored by held-out bits per byte.

Config (the byte-level LM of the benchmark set): 4 layers, d 256, 4 heads, ctx 256, vocabulary 256,
pre-RMSNorm, RoPE, GELU MLP 4x; AdamW lr 3e-4, weight decay 0.1; batch 64; tokens are seeded i.i.d.
bytes from a Zipf(1.1) law over 256 symbols.  Bits per byte follows the reference's definition
(PredictiveCoding.LLM/PredictiveLlm.cs:485-500): non-overlapping windows of min(32, ctx) tokens, total
NLL / ln 2 divided by the bytes of the targets; every token here is one byte.  The held-out stream has
its own seed.  The two runs differ only in the arithmetic of their kernels and in where AdamW applies
decay (the reference's order, after the step, in the fused trainer; torch's, before it, in the baseline).

    python -m predicitivecoding_b200.bench_bytelm --steps 300
"""
from __future__ import annotations

import argparse
import copy
import json
import math
import time

import torch


def held_out_bpb(model, tokens: torch.Tensor, window: int = 32, device="cuda") -> float:
    """Mean NLL / ln 2 per target byte over non-overlapping windows of ``window`` tokens (fp32 forward)."""
    model = model.to(device).float().eval()
    n = (tokens.numel() - 1) // window
    x = tokens[: n * window].view(n, window).to(device)
    y = tokens[1: n * window + 1].view(n, window).to(device)
    nll = 0.0
    with torch.no_grad():
        for i in range(0, n, 256):
            logits = model(x[i:i + 256]).float()
            nll += float(torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]),
                                                           y[i:i + 256].reshape(-1), reduction="sum"))
    return nll / math.log(2) / (n * window)


def run(steps: int = 300, batch: int = 64, seed: int = 42, device="cuda") -> dict:
    from .engine.fused_trainer import FusedDecoderTrainer
    from .models.config import DecoderLmConfig
    from .models.decoder_lm import DecoderLM
    from .utils.data import zipf_tokens, zipf_windows

    cfg = DecoderLmConfig.byte_lm_4l()
    S = cfg.max_seq
    init = DecoderLM(cfg, seed=seed)
    fused = FusedDecoderTrainer(cfg, batch, S, device=device, lr=3e-4, weight_decay=0.1, model=copy.deepcopy(init))
    base = copy.deepcopy(init).to(device)
    opt = torch.optim.AdamW(base.parameters(), lr=3e-4, weight_decay=0.1, fused=True)
    losses_f, losses_t = [], []
    t0 = time.perf_counter()
    for step in range(steps):
        tok, tgt = zipf_windows(batch, S, cfg.vocab, 1.1, seed=10_000 + step)
        losses_f.append(fused.step(tok, tgt))
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = base(tok.to(device))
            loss = torch.nn.functional.cross_entropy(logits.float().view(-1, cfg.vocab), tgt.to(device).view(-1))
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses_t.append(float(loss))
    train_s = time.perf_counter() - t0
    held = zipf_tokens(64 * 32 * 32 + 1, cfg.vocab, 1.1, seed=987_654)
    bpb_f = held_out_bpb(fused.export_model(), held, device=device)
    bpb_t = held_out_bpb(base, held, device=device)
    p = torch.arange(1, cfg.vocab + 1, dtype=torch.float64) ** -1.1
    p /= p.sum()
    entropy_bits = float(-(p * torch.log2(p)).sum())
    return {"metric": "byte-LM held-out bits per byte (fused trainer vs PyTorch baseline, same init and batches)",
            "steps": steps, "batch": batch, "seq_len": S,
            "bpb_fused": round(bpb_f, 4), "bpb_torch": round(bpb_t, 4),
            "relative_difference": round(abs(bpb_f - bpb_t) / bpb_t, 5),
            "source_entropy_bits": round(entropy_bits, 4),
            "final_train_loss_fused": round(sum(losses_f[-10:]) / 10, 4),
            "final_train_loss_torch": round(sum(losses_t[-10:]) / 10, 4),
            "wall_seconds_both": round(train_s, 1),
            "data": "synthetic (seeded Zipf(1.1) bytes; held-out stream with its own seed)",
            "dtype": "bf16 compute, fp32 master weights (both)"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--batch", type=int, default=64)
    a = ap.parse_args()
    print(json.dumps(run(a.steps, a.batch)))


if __name__ == "__main__":
    main()

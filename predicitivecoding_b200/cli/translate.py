"""Translation CLI: gradcheck, smoke, train, train-tatoeba, translate.

Reference: PredictiveCoding.Translate.Cli/Program.cs:9-340 (``--key value`` argument map;
gradcheck = central-difference check of the masked cross-entropy and of the decoder's gradients;
smoke = tiny train + translate; train = BPE on prompt+target lines, examples longer than --maxseq
dropped, warmup + cosine AdamW, periodic samples, save to --out; translate = load --model and
translate --text into --to).  Training runs on the GPU when one is present.
"""
from __future__ import annotations

import math
import random
import sys
from typing import Dict, List

import torch

from ..llm import translation as tr
from ..models.config import DecoderLmConfig
from ..models.decoder_lm import DecoderLM, cross_entropy_masked
from ..optim.adam import Adam, LrSchedule
from ..llm.trainer import step as adam_step


def arg_map(argv: List[str]) -> Dict[str, str]:
    d: Dict[str, str] = {}
    i = 0
    while i < len(argv):
        if argv[i].startswith("--"):
            key = argv[i][2:]
            if i + 1 < len(argv) and not argv[i + 1].startswith("--"):
                d[key] = argv[i + 1]
                i += 1
            else:
                d[key] = "true"
        i += 1
    return d


def _num(a, k, d, cast=int):
    return cast(a[k]) if k in a else d


def gradcheck(eps: float = 1e-3, seed: int = 0) -> bool:
    """Central differences vs autograd on the masked CE and on a tiny decoder (float64)."""
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(5, 7, generator=g, dtype=torch.float64, requires_grad=True)
    tgt = torch.tensor([1, -1, 3, 6, 0])
    loss = cross_entropy_masked(logits, tgt, -1)
    loss.backward()
    num = torch.zeros_like(logits)
    with torch.no_grad():
        for idx in range(logits.numel()):
            x = logits.detach().clone().reshape(-1)
            x[idx] += eps
            lp = cross_entropy_masked(x.view_as(logits), tgt, -1)
            x[idx] -= 2 * eps
            lm = cross_entropy_masked(x.view_as(logits), tgt, -1)
            num.view(-1)[idx] = (lp - lm) / (2 * eps)
    ok_ce = torch.allclose(num, logits.grad, atol=1e-6, rtol=1e-4)
    m = DecoderLM(DecoderLmConfig(16, 8, 1, 2, 16, 8), seed=seed).double()
    t = torch.randint(0, 16, (1, 6), generator=g)
    y = torch.randint(0, 16, (1, 6), generator=g)
    m.loss(t, y, -1, False).backward()
    p = m.wemb
    worst = 0.0
    with torch.no_grad():
        for idx in range(0, p.numel(), max(1, p.numel() // 24)):
            flat = p.view(-1)
            old = float(flat[idx])
            flat[idx] = old + eps
            lp = float(m.loss(t, y, -1, False))
            flat[idx] = old - eps
            lm = float(m.loss(t, y, -1, False))
            flat[idx] = old
            worst = max(worst, abs((lp - lm) / (2 * eps) - float(p.grad.view(-1)[idx])))
    ok_model = worst < 1e-5
    print(f"gradcheck: masked CE {'PASS' if ok_ce else 'FAIL'}, decoder max |delta| {worst:.2e} "
          f"{'PASS' if ok_model else 'FAIL'}")
    return ok_ce and ok_model


def run_training(a: Dict[str, str], pairs=None) -> int:
    corpus = a.get("corpus")
    if pairs is None:
        if corpus is None:
            print("error: --corpus <path.tsv> is required", file=sys.stderr)
            return 2
        pairs = list(tr.read_tsv(corpus))
    limit = _num(a, "limit", 0)
    if limit:
        pairs = pairs[:limit]
    dim, blocks, heads = _num(a, "dim", 256), _num(a, "blocks", 4), _num(a, "heads", 4)
    ff, max_seq, merges = _num(a, "ff", dim * 4), _num(a, "maxseq", 96), _num(a, "merges", 8000)
    epochs, batch, lr = _num(a, "epochs", 1), _num(a, "batch", 16), _num(a, "lr", 3e-4, float)
    out = a.get("out", "translator-out")
    tok = tr.train_tokenizer(pairs, merges)
    ex = tr.build_examples(pairs, tok, max_seq)
    if not ex:
        print("error: every example exceeds --maxseq", file=sys.stderr)
        return 2
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    model = DecoderLM(DecoderLmConfig(tok.vocab_size, dim, blocks, heads, ff, max_seq), seed=42).to(dev)
    opt = Adam(weight_decay=0.01)
    steps = max(1, epochs * math.ceil(len(ex) / batch))
    sched = LrSchedule(lr, lr * 0.1, max(1, steps // 10), steps)
    rng = random.Random(7)
    k = 0
    for _ in range(epochs):
        rng.shuffle(ex)
        for i in range(0, len(ex), batch):
            loss = adam_step(list(model.parameters()), ex[i:i + batch],
                             lambda t, y, trn: model.loss(t.view(1, -1), y.view(1, -1), -1, trn), opt, sched.at(k), 1.0)
            k += 1
            if k % _num(a, "sample-every", 200) == 0:
                print(f"step {k}/{steps} loss {loss:.4f}")
    t = tr.Translator(model.cpu(), tok)
    t.save(out)
    print(f"saved translator to {out}")
    return 0


def smoke() -> int:
    pairs = [tr.SentencePair(s, t, "it") for s, t in
             [("hello", "ciao"), ("cat", "gatto"), ("dog", "cane"), ("house", "casa")]] * 8
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        rc = run_training({"dim": "32", "blocks": "1", "heads": "2", "maxseq": "32", "merges": "40", "epochs": "30",
                           "batch": "8", "lr": "0.01", "out": d, "sample-every": "1000000"}, pairs)
        out = tr.Translator.load(d).translate("cat", "it", 8)
    print(f"smoke: 'cat' -> '{out}'")
    return rc


def translate(a: Dict[str, str]) -> int:
    if "model" not in a or "text" not in a:
        print("usage: translate --model <dir> --text <source> [--to it]", file=sys.stderr)
        return 2
    print(tr.Translator.load(a["model"]).translate(a["text"], a.get("to", "it"), _num(a, "max", 64)))
    return 0


def main(argv: List[str] = None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if not argv or argv[0] in ("help", "--help", "-h"):
        print("commands: gradcheck | smoke | train --corpus f.tsv [--out dir ...] | train-tatoeba --corpus f.tsv | "
              "translate --model dir --text '...' [--to tag]")
        return 0
    cmd, a = argv[0], arg_map(argv[1:])
    if cmd == "gradcheck":
        return 0 if gradcheck() else 1
    if cmd == "smoke":
        return smoke()
    if cmd in ("train", "train-tatoeba"):
        if cmd == "train-tatoeba":
            a.setdefault("merges", "16000")
        return run_training(a)
    if cmd == "translate":
        return translate(a)
    print(f"unknown command {cmd!r}", file=sys.stderr)
    return 2


if __name__ == "__main__":
    sys.exit(main())

"""Evaluation: perplexity, held-out splits (positional and content-hashed), bits per byte,
activation probes, regression baselines and the HTML report.

Reference: PredictiveCoding.LLM/Eval/PerplexityEvaluator.cs:25-140 (token-weighted NLL,
positional split every k-th window, FNV-1a content hash split), PredictiveLlm.cs:485-500
(bits-per-byte: non-overlapping windows of min(32, MaxSeq) tokens, total NLL / ln 2 divided
by the UTF-8 bytes of the decoded scored targets), Eval/ActivationProbe.cs:18-81,
Eval/RegressionHarness.cs, Eval/HtmlReport.cs.
"""
from __future__ import annotations

import html
import json
import math
import os
from dataclasses import asdict, dataclass, field
from typing import Dict, Iterable, Iterator, List, Optional, Sequence, Tuple

import torch

from .data import StreamingTextDataset

Window = Tuple[Sequence[int], Sequence[int]]


@dataclass(frozen=True)
class PerplexityResult:
    perplexity: float
    nll_per_token: float
    tokens: int
    windows: int


@dataclass(frozen=True)
class BitsPerByteResult:
    bits_per_byte: float
    bytes: int
    tokens: int


def fnv1a_tokens(tokens: Sequence[int]) -> int:
    """FNV-1a 32-bit over the little-endian bytes of each token id (PerplexityEvaluator.cs:118-129)."""
    h = 2166136261
    for t in tokens:
        v = int(t) & 0xFFFFFFFF
        for b in range(4):
            h ^= (v >> (8 * b)) & 0xFF
            h = (h * 16777619) & 0xFFFFFFFF
    return h


def held_out(windows: Iterable[Window], every: int = 10) -> Iterator[Window]:
    if every < 2:
        raise ValueError("every must be >= 2.")
    for i, w in enumerate(windows):
        if i % every == 0:
            yield w


def training_split(windows: Iterable[Window], every: int = 10) -> Iterator[Window]:
    if every < 2:
        raise ValueError("every must be >= 2.")
    for i, w in enumerate(windows):
        if i % every != 0:
            yield w


def held_out_hashed(windows: Iterable[Window], every: int = 10) -> Iterator[Window]:
    if every < 2:
        raise ValueError("every must be >= 2.")
    for w in windows:
        if fnv1a_tokens(w[0]) % every == 0:
            yield w


def training_split_hashed(windows: Iterable[Window], every: int = 10) -> Iterator[Window]:
    if every < 2:
        raise ValueError("every must be >= 2.")
    for w in windows:
        if fnv1a_tokens(w[0]) % every != 0:
            yield w


@torch.no_grad()
def evaluate(model, windows: Iterable[Window], ignore_index: int = -1, max_windows: Optional[int] = None,
             device=None, batch: int = 64) -> PerplexityResult:
    """Token-weighted mean NLL over the windows (training=False forward, fp32 log-sum-exp)."""
    device = device or next(model.parameters()).device
    nll, tokens, used = 0.0, 0, 0
    buf: List[Window] = []

    def flush():
        nonlocal nll, tokens
        if not buf:
            return
        L = max(len(w[0]) for w in buf)
        same = all(len(w[0]) == L for w in buf)
        groups = [buf] if same else [[w] for w in buf]
        for g in groups:
            x = torch.tensor([list(w[0]) for w in g], device=device)
            y = torch.tensor([list(w[1]) for w in g], device=device)
            logits = model.forward(x).float()
            lp = torch.log_softmax(logits, -1)
            keep = y != ignore_index
            nll += float(-(lp.gather(-1, y.clamp(min=0).unsqueeze(-1)).squeeze(-1) * keep).sum())
            tokens += int(keep.sum())
        buf.clear()

    for w in windows:
        if max_windows is not None and used >= max_windows:
            break
        buf.append(w)
        used += 1
        if len(buf) >= batch:
            flush()
    flush()
    if tokens == 0:
        raise RuntimeError("No scorable tokens: the window stream was empty or every target is ignore_index.")
    per = nll / tokens
    return PerplexityResult(math.exp(min(per, 700.0)), per, tokens, used)


def bits_per_byte(model, tokenizer, text: str, max_seq: int, fallback_window=None) -> BitsPerByteResult:
    """Tokenizer-independent yardstick (PredictiveLlm.cs:485-500)."""
    seq = min(32, max_seq)
    windows = list(StreamingTextDataset(text.split("\n"), tokenizer, seq, seq).windows())
    if not windows:
        if fallback_window is None:
            raise RuntimeError("Text too short to evaluate.")
        windows = [fallback_window]
    ppl = evaluate(model, windows)
    nbytes = sum(len(tokenizer.decode(t).encode("utf-8")) for _, t in windows)
    total_bits = ppl.nll_per_token * ppl.tokens / math.log(2)
    return BitsPerByteResult(total_bits / max(1, nbytes), nbytes, ppl.tokens)


class ActivationProbe:
    """Per-block activation statistics and attention-sink shares (Eval/ActivationProbe.cs:18-81)."""

    def __init__(self):
        self.blocks: Dict[int, Dict[str, float]] = {}
        self.sink_share: Dict[int, float] = {}
        self.loops_used = 0
        self.moe_rows_computed = 0

    def record_block(self, index: int, x: torch.Tensor) -> None:
        a = x.detach().float().abs()
        self.blocks[index] = {"mean_abs": float(a.mean()), "max_abs": float(a.max())}

    def record_causal_attention(self, block: int, probs: torch.Tensor) -> None:
        # share of attention mass on position 0 (the "sink"), averaged over heads and queries
        self.sink_share[block] = float(probs[..., 0].float().mean())

    def to_dict(self) -> Dict:
        return {"blocks": self.blocks, "sink_share": self.sink_share, "loops_used": self.loops_used,
                "moe_rows_computed": self.moe_rows_computed}


class RegressionHarness:
    """JSON baseline of named metrics with a relative-tolerance diff (Eval/RegressionHarness.cs)."""

    def __init__(self, path: str, rel_tol: float = 0.02):
        self.path, self.rel_tol = path, rel_tol

    def save(self, metrics: Dict[str, float]) -> None:
        with open(self.path, "w") as f:
            json.dump(metrics, f, indent=2, sort_keys=True)

    def compare(self, metrics: Dict[str, float]) -> Dict[str, Tuple[float, float, bool]]:
        base = json.load(open(self.path)) if os.path.exists(self.path) else {}
        out = {}
        for k, v in metrics.items():
            if k in base:
                b = base[k]
                ok = abs(v - b) <= self.rel_tol * max(abs(b), 1e-12)
                out[k] = (b, v, ok)
        return out


TINY_EVAL_CORPUS = (
    "The quick brown fox jumps over the lazy dog.\n"
    "Predictive coding networks minimise prediction error layer by layer.\n"
    "A language model assigns probabilities to the next token of a sequence.\n"
    "Bits per byte compares models with different tokenizers on the same text.\n"
)


def html_report(path: str, title: str, ppl: PerplexityResult, probe: Optional[ActivationProbe] = None,
                extra: Optional[Dict] = None) -> str:
    """Self-contained HTML report (Eval/HtmlReport.cs); returns the path written."""
    rows = "".join(f"<tr><td>{html.escape(str(k))}</td><td>{html.escape(json.dumps(v))}</td></tr>"
                   for k, v in {**asdict(ppl), **(extra or {})}.items())
    probe_html = ""
    if probe is not None:
        brow = "".join(f"<tr><td>{b}</td><td>{s['mean_abs']:.4f}</td><td>{s['max_abs']:.4f}</td>"
                       f"<td>{probe.sink_share.get(b, float('nan')):.3f}</td></tr>" for b, s in sorted(probe.blocks.items()))
        probe_html = ("<h2>Activations</h2><table><tr><th>block</th><th>mean|a|</th><th>max|a|</th>"
                      f"<th>sink share</th></tr>{brow}</table>")
    doc = (f"<!doctype html><html><head><meta charset='utf-8'><title>{html.escape(title)}</title>"
           "<style>body{font-family:sans-serif}td,th{padding:2px 8px;border-bottom:1px solid #ddd}</style>"
           f"</head><body><h1>{html.escape(title)}</h1><table>{rows}</table>{probe_html}</body></html>")
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "w", encoding="utf-8") as f:
        f.write(doc)
    return path


# ---------------------------------------------------------------- fixed yardstick text + multi-metric bundle
# A small, fixed text written for this package so that perplexities quoted by tests and demos are
# always measured on the same bytes (Eval/EvalCorpus.cs plays this role in the reference, with its own
# text; the two corpora differ, so their numbers are not comparable).
EVAL_CORPUS_LINES = (
    "Rivers carry the memory of rain down to the sea.",
    "A map is a guess about a territory that keeps changing.",
    "Each morning the baker checks whether the dough has risen as expected.",
    "When the forecast is wrong, the sailor trims the sails and watches the sky.",
    "Small surprises teach more than large certainties.",
    "The orchestra listens to itself and corrects the tempo bar by bar.",
    "Rivers carry the memory of rain down to the sea.",
    "A good guess saves words, and saved words make a short message.",
    "The lighthouse keeper counts ships and notes the ones that never arrive.",
    "Small surprises teach more than large certainties.",
)


def eval_corpus() -> str:
    return "\n".join(EVAL_CORPUS_LINES)


@dataclass(frozen=True)
class ProbeScores:
    echo: float
    induction: float


@dataclass(frozen=True)
class ProEvalReport:
    bits_per_byte: BitsPerByteResult
    per_domain_perplexity: Dict[str, float]
    probes: ProbeScores
    serve_tokens_per_second: float


def next_token_accuracy(llm, text: str) -> float:
    """Share of positions whose greedy next token equals the text's next token."""
    ids = llm.tokenizer.encode(text)
    n = min(len(ids), llm.config.max_seq)
    if n < 2:
        return 0.0
    tokens = torch.tensor(ids[:n], dtype=torch.long, device=next(llm.model.parameters()).device)
    with torch.no_grad():
        pred = llm.model(tokens).argmax(-1)
    return float((pred[:-1] == tokens[1:]).float().mean())


def pro_eval(llm, reference_text: str, domains: Dict[str, str], serve_tokens: int = 32) -> ProEvalReport:
    """Bits per byte on a reference text, perplexity per domain, two in-context probes (echo: a
    repeated token; induction: a repeated pair) and generation throughput (ProEval.cs:8-100)."""
    import time
    if not reference_text:
        raise ValueError("reference_text must not be empty")
    bpb = llm.evaluate_bits_per_byte(reference_text)
    per = {name: llm.evaluate(text).perplexity for name, text in domains.items()}
    probes = ProbeScores(next_token_accuracy(llm, "A " * 24), next_token_accuracy(llm, "A B " * 16))
    prompt = reference_text[:24]
    llm.generate(prompt, max_new_tokens=4)
    t0 = time.perf_counter()
    llm.generate(prompt, max_new_tokens=serve_tokens)
    dt = time.perf_counter() - t0
    return ProEvalReport(bpb, per, probes, serve_tokens / dt if dt > 0 else 0.0)


# --------------------------------------------------------------------------- KV-cache model loss
def token_loss(logits: torch.Tensor, target: int) -> float:
    """-log softmax(logits)[target] with a max-shifted log-sum-exp (CrossEntropy.cs:17-27)."""
    l = logits.detach().double().reshape(-1)
    return float(torch.logsumexp(l, 0) - l[target])


@torch.no_grad()
def evaluate_gpt(model, tokens) -> tuple:
    """Teacher-forced mean next-token cross-entropy and perplexity exp(loss) of a KV-cache model
    (``GptModel.step``) over one token sequence, stopping at the context limit (CrossEntropy.cs:33-52).
    Returns (0, 1) for fewer than two tokens."""
    tokens = list(tokens)
    if len(tokens) < 2:
        return 0.0, 1.0
    cache = model.create_cache()
    total, count, pos = 0.0, 0, 0
    for i in range(len(tokens) - 1):
        if pos >= model.max_seq_len:
            break
        logits = model.step(tokens[i], pos, cache)
        pos += 1
        total += token_loss(logits, tokens[i + 1])
        count += 1
    loss = total / count if count else 0.0
    return loss, math.exp(loss)

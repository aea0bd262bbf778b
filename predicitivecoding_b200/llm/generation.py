"""Decoding: sampler, greedy / self-speculative decoding, beam search, batched lockstep
generation, continuous batching and chat templates.

Reference: PredictiveCoding.LLM/Generation/Sampling.cs:13-148 (temperature, top-k, top-p,
repetition/presence/frequency penalties, greedy, seeded RNG), SelfSpeculative.cs:17-122
(the t+2 multi-token head drafts, the next forward verifies: output identical to greedy),
BeamSearch.cs, BatchedGenerator.cs, ContinuousBatcher.cs:18-113, ChatTemplate.cs.
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch


@dataclass(frozen=True)
class SamplingOptions:
    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 1.0
    repetition_penalty: float = 1.0
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    greedy: bool = False
    max_new_tokens: int = 128
    seed: Optional[int] = None


class Sampler:
    """Turns next-token logits into a token id (Sampling.cs:41-148)."""

    def __init__(self, seed: Optional[int] = None):
        self.rng = random.Random(seed)

    def sample(self, logits: torch.Tensor, generated: Sequence[int], o: SamplingOptions) -> int:
        l = logits.detach().float().cpu().clone()
        if (o.repetition_penalty != 1.0 or o.presence_penalty != 0.0 or o.frequency_penalty != 0.0) and generated:
            counts: Dict[int, int] = {}
            for t in generated:
                if 0 <= t < l.numel():
                    counts[t] = counts.get(t, 0) + 1
            for t, c in counts.items():
                if o.repetition_penalty != 1.0:
                    l[t] = l[t] / o.repetition_penalty if l[t] > 0 else l[t] * o.repetition_penalty
                l[t] -= o.presence_penalty + o.frequency_penalty * c
        if o.greedy:
            return int(torch.argmax(l))
        l = l / max(o.temperature, 1e-5)
        p = torch.softmax(l, -1)
        if 0 < o.top_k < p.numel():
            thr = torch.sort(p).values[p.numel() - o.top_k]
            p = torch.where(p < thr, torch.zeros_like(p), p)
        if o.top_p < 1.0:
            order = torch.argsort(p, descending=True)
            cum, kept = 0.0, False
            for i in order.tolist():
                if kept and cum >= o.top_p:
                    p[i] = 0.0
                    continue
                cum += float(p[i])
                kept = True
        s = float(p.sum())
        p = p / s if s > 0 else torch.full_like(p, 1.0 / p.numel())
        r = self.rng.random()
        acc = 0.0
        for i, pi in enumerate(p.tolist()):
            acc += pi
            if r <= acc:
                return i
        return p.numel() - 1


@dataclass
class SpeculativeResult:
    tokens: List[int]
    forwards: int
    drafted: int
    accepted: int

    @property
    def acceptance_rate(self) -> float:
        return self.accepted / self.drafted if self.drafted else 0.0


def _fwd_heads(model, seq: List[int]):
    t = torch.tensor(seq, device=model.wemb.device)
    with torch.no_grad():
        main, mtp = model.heads(t)
    return main, mtp


@torch.no_grad()
def greedy(model, prompt: Sequence[int], max_new_tokens: int, eos: int = -1) -> List[int]:
    seq = list(prompt)
    for _ in range(max_new_tokens):
        if len(seq) >= model.cfg.max_seq:
            break
        logits = model.forward(torch.tensor(seq, device=model.wemb.device))
        seq.append(int(torch.argmax(logits[-1])))
        if seq[-1] == eos:
            break
    return seq


@torch.no_grad()
def self_speculative(model, prompt: Sequence[int], max_new_tokens: int, eos: int = -1) -> SpeculativeResult:
    """Greedy decoding that uses the t+2 head as a drafter; identical output to greedy()."""
    seq = list(prompt)
    max_seq = model.cfg.max_seq
    generated = forwards = drafted = accepted = 0
    pending = -1
    while generated < max_new_tokens and len(seq) < max_seq:
        if pending >= 0 and len(seq) + 1 <= max_seq:
            seq.append(pending)
            main, mtp = _fwd_heads(model, seq)
            forwards += 1
            real = int(torch.argmax(main[len(seq) - 2]))
            if real == pending:
                accepted += 1
                generated += 1
                if seq[-1] == eos or generated >= max_new_tokens or len(seq) >= max_seq:
                    break
                seq.append(int(torch.argmax(main[len(seq) - 1])))
                generated += 1
                if seq[-1] == eos:
                    break
                pending = int(torch.argmax(mtp[len(seq) - 2]))
                drafted += 1
            else:
                seq[-1] = real
                generated += 1
                if real == eos:
                    break
                pending = int(torch.argmax(mtp[len(seq) - 2]))
                drafted += 1
        else:
            pending = -1
            main, mtp = _fwd_heads(model, seq)
            forwards += 1
            seq.append(int(torch.argmax(main[len(seq) - 1])))
            generated += 1
            if seq[-1] == eos:
                break
            if mtp is not None:
                pending = int(torch.argmax(mtp[len(seq) - 2]))
                drafted += 1
    return SpeculativeResult(seq, forwards, drafted, accepted)


@torch.no_grad()
def beam_search(step_logprobs: Callable[[List[int]], torch.Tensor], prompt: Sequence[int], beam_width: int,
                max_new_tokens: int, eos: int = -1, length_penalty: float = 1.0) -> List[int]:
    """Beam search over a next-token log-prob function (Generation/BeamSearch.cs)."""
    beams = [(0.0, list(prompt), False)]
    for _ in range(max_new_tokens):
        cand = []
        for score, seq, done in beams:
            if done:
                cand.append((score, seq, True))
                continue
            lp = step_logprobs(seq)
            top = torch.topk(lp, beam_width)
            for v, i in zip(top.values.tolist(), top.indices.tolist()):
                cand.append((score + v, seq + [i], i == eos))
        cand.sort(key=lambda c: c[0] / (max(1, len(c[1]) - len(prompt)) ** length_penalty), reverse=True)
        beams = cand[:beam_width]
        if all(d for _, _, d in beams):
            break
    return beams[0][1]


class ChatTemplate:
    """Role-tagged prompt format (Generation/ChatTemplate.cs): <|system|> / <|user|> / <|assistant|>."""

    @staticmethod
    def format(system: Optional[str], turns: Sequence[Tuple[str, str]], add_generation_prompt: bool = True) -> str:
        parts = []
        if system:
            parts.append(f"<|system|>\n{system}\n")
        for role, text in turns:
            parts.append(f"<|{role}|>\n{text}\n")
        if add_generation_prompt:
            parts.append("<|assistant|>\n")
        return "".join(parts)


@dataclass
class _Slot:
    id: int
    tokens: List[int]
    prompt_len: int
    max_new: int
    done: bool = False


class ContinuousBatcher:
    """Admits requests into free slots, decodes all active slots in lockstep, evicts finished ones
    (Generation/ContinuousBatcher.cs:18-113).  ``decode_fn(list of sequences) -> next-token ids``."""

    def __init__(self, decode_fn: Callable[[List[List[int]]], List[int]], slots: int, eos: int = -1):
        self.decode_fn, self.capacity, self.eos = decode_fn, slots, eos
        self.active: List[_Slot] = []
        self.queue: List[_Slot] = []
        self.finished: Dict[int, List[int]] = {}
        self._next = 0

    def submit(self, prompt: Sequence[int], max_new_tokens: int) -> int:
        s = _Slot(self._next, list(prompt), len(prompt), max_new_tokens)
        self._next += 1
        self.queue.append(s)
        return s.id

    def step(self) -> None:
        while self.queue and len(self.active) < self.capacity:
            self.active.append(self.queue.pop(0))
        if not self.active:
            return
        nxt = self.decode_fn([s.tokens for s in self.active])
        for s, t in zip(self.active, nxt):
            s.tokens.append(int(t))
            if int(t) == self.eos or len(s.tokens) - s.prompt_len >= s.max_new:
                s.done = True
        for s in [s for s in self.active if s.done]:
            self.finished[s.id] = s.tokens[s.prompt_len:]
            self.active.remove(s)

    def run(self) -> Dict[int, List[int]]:
        while self.queue or self.active:
            self.step()
        return self.finished


def _prefill(model, prompt: Sequence[int], cache, bos: int):
    """Feed the prompt (a lone BOS when empty) one position at a time; returns (logits, next position)."""
    prompt = list(prompt) if len(prompt) > 0 else [bos]
    pos = 0
    logits = model.step(prompt[0], pos, cache)
    pos += 1
    for t in prompt[1:]:
        if pos >= model.max_seq_len:
            break
        logits = model.step(t, pos, cache)
        pos += 1
    return logits, pos, prompt


class TextGenerator:
    """Autoregressive generation over a KV-cache model (TextGenerator.cs:16-70): prefill the prompt, then
    sample, append and decode-step until EOS, ``max_new_tokens`` or the context is full."""

    def __init__(self, model, tokenizer):
        self.model, self.tokenizer = model, tokenizer

    def generate(self, prompt: str, options: SamplingOptions, on_token: Optional[Callable[[int], None]] = None) -> str:
        ids = self.generate_tokens(self.tokenizer.encode(prompt, add_bos=True), options, on_token)
        return self.tokenizer.decode(ids)

    @torch.no_grad()
    def generate_tokens(self, prompt: Sequence[int], options: SamplingOptions,
                        on_token: Optional[Callable[[int], None]] = None) -> List[int]:
        m = self.model
        cache = m.create_cache()
        sampler = Sampler(options.seed)
        logits, pos, ctx = _prefill(m, prompt, cache, self.tokenizer.bos)
        context = list(ctx)
        out: List[int] = []
        for _ in range(options.max_new_tokens):
            if pos >= m.max_seq_len:
                break
            nxt = sampler.sample(logits, context, options)
            if nxt == self.tokenizer.eos:
                break
            out.append(nxt)
            context.append(nxt)
            if on_token is not None:
                on_token(nxt)
            logits = m.step(nxt, pos, cache)
            pos += 1
        return out


class BatchedGenerator:
    """Several independent prompts decoded in lockstep (BatchedGenerator.cs:16-83): every sequence has its
    own KV cache and sampler (seed + i), and the loop advances all live sequences one token per step until
    each hits EOS, ``max_new_tokens`` or the context limit."""

    def __init__(self, model, tokenizer):
        self.model, self.tokenizer = model, tokenizer

    def generate(self, prompts: Sequence[str], options: SamplingOptions) -> List[str]:
        enc = [self.tokenizer.encode(p, add_bos=True) for p in prompts]
        return [self.tokenizer.decode(t) for t in self.generate_batch(enc, options)]

    @torch.no_grad()
    def generate_batch(self, prompts: Sequence[Sequence[int]], options: SamplingOptions) -> List[List[int]]:
        m, n = self.model, len(prompts)
        caches = [m.create_cache() for _ in range(n)]
        samplers = [Sampler(None if options.seed is None else options.seed + i) for i in range(n)]
        logits, pos, context = [None] * n, [0] * n, [None] * n
        for i in range(n):
            logits[i], pos[i], ctx = _prefill(m, prompts[i], caches[i], self.tokenizer.bos)
            context[i] = list(ctx)
        out: List[List[int]] = [[] for _ in range(n)]
        done = [False] * n
        for _ in range(options.max_new_tokens):
            active = False
            for i in range(n):
                if done[i]:
                    continue
                active = True
                nxt = samplers[i].sample(logits[i], context[i], options)
                if nxt == self.tokenizer.eos or pos[i] >= m.max_seq_len:
                    done[i] = True
                    continue
                out[i].append(nxt)
                context[i].append(nxt)
                logits[i] = m.step(nxt, pos[i], caches[i])
                pos[i] += 1
            if not active:
                break
        return out

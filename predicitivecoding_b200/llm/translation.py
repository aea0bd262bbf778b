"""Tagged-prompt translation on the decoder: corpus reading, example building, greedy/sampled decode,
and a self-contained save/load folder (manifest + BPE tokenizer + weights).

Reference: PredictiveCoding.LLM/Translation/TranslationFormat.cs:1-70 (prompt ``>>tag<< source\\n``,
examples [BOS] prompt target [EOS] with the prompt's targets ignored), ParallelCorpus.cs:1-63 (TSV
tag/src/tgt with '#' comments; tokenizer trained on prompt+target lines; examples longer than
max_seq dropped) and Translator.cs:1-126 (decode until EOS or max_seq; manifest.json,
tokenizer.bpe, weights/).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import Iterable, List, Optional, Tuple

import torch

from ..io import checkpoint as ck
from ..models.config import DecoderLmConfig
from ..models.decoder_lm import DecoderLM
from .tokenizer import BpeTokenizer

IGNORE_INDEX = -1


@dataclass(frozen=True)
class SentencePair:
    source: str
    target: str
    target_tag: str


def prompt_text(source: str, tag: str) -> str:
    return f">>{tag}<< {source}\n"


def build_example(tok: BpeTokenizer, source: str, target: str, tag: str) -> Tuple[List[int], List[int]]:
    p = tok.encode(prompt_text(source, tag))
    full = [tok.bos] + p + tok.encode(target) + [tok.eos]
    tokens, targets = full[:-1], full[1:]
    for i in range(len(p)):
        targets[i] = IGNORE_INDEX
    return tokens, targets


def build_prompt(tok: BpeTokenizer, source: str, tag: str) -> List[int]:
    return [tok.bos] + tok.encode(prompt_text(source, tag))


def read_tsv(path: str, tag_col: int = 0, src_col: int = 1, tgt_col: int = 2, sep: str = "\t"):
    need = max(tag_col, src_col, tgt_col)
    for line in open(path, encoding="utf-8"):
        line = line.rstrip("\n")
        if not line.strip() or line[0] == "#":
            continue
        cols = line.split(sep)
        if len(cols) <= need:
            continue
        tag, src, tgt = cols[tag_col].strip(), cols[src_col].strip(), cols[tgt_col].strip()
        if tag and src and tgt:
            yield SentencePair(src, tgt, tag)


def train_tokenizer(pairs: Iterable[SentencePair], merges: int) -> BpeTokenizer:
    text = "".join(prompt_text(p.source, p.target_tag) + p.target + "\n" for p in pairs)
    tok = BpeTokenizer()
    tok.train(text, merges)
    return tok


def build_examples(pairs: Iterable[SentencePair], tok: BpeTokenizer, max_seq: int):
    out = []
    for p in pairs:
        ex = build_example(tok, p.source, p.target, p.target_tag)
        if len(ex[0]) <= max_seq:
            out.append(ex)
    return out


class Translator:
    MANIFEST, TOKENIZER, WEIGHTS = "manifest.json", "tokenizer.bpe", "weights"

    def __init__(self, model: DecoderLM, tok: BpeTokenizer):
        self.model, self.tok = model, tok

    @property
    def config(self) -> DecoderLmConfig:
        return self.model.cfg

    @torch.no_grad()
    def translate(self, source: str, tag: str, max_new_tokens: int = 256, temperature: float = 0.0,
                  gen: Optional[torch.Generator] = None) -> str:
        seq = build_prompt(self.tok, source, tag)
        out = []
        dev = next(self.model.parameters()).device
        self.model.eval()
        while len(out) < max_new_tokens and len(seq) < self.config.max_seq:
            row = self.model(torch.tensor([seq], device=dev))[0, -1].float().cpu()
            if temperature <= 0:
                nxt = int(row.argmax())
            else:
                nxt = int(torch.multinomial(torch.softmax(row / temperature, -1), 1, generator=gen))
            if nxt == self.tok.eos:
                break
            seq.append(nxt)
            out.append(nxt)
        return self.tok.decode(out).strip()

    def save(self, d: str) -> None:
        os.makedirs(d, exist_ok=True)
        c = self.config
        with open(os.path.join(d, self.MANIFEST), "w") as f:
            json.dump({"Vocab": c.vocab, "Dim": c.dim, "NumBlocks": c.num_blocks, "NumHeads": c.num_heads,
                       "FfDim": c.ff_dim, "MaxSeq": c.max_seq, "Eps": c.eps}, f, indent=2)
        self.tok.save(os.path.join(d, self.TOKENIZER))
        ck.save_parameters(os.path.join(d, self.WEIGHTS), self.model.reference_parameters())

    @staticmethod
    def load(d: str) -> "Translator":
        m = json.load(open(os.path.join(d, Translator.MANIFEST)))
        cfg = DecoderLmConfig(m["Vocab"], m["Dim"], m["NumBlocks"], m["NumHeads"], m["FfDim"], m["MaxSeq"],
                              dropout=0.0, eps=m["Eps"])
        tok = BpeTokenizer.load(os.path.join(d, Translator.TOKENIZER))
        model = DecoderLM(cfg, seed=0)
        model.load_reference_parameters(ck.load_parameters(os.path.join(d, Translator.WEIGHTS)))
        return Translator(model, tok)

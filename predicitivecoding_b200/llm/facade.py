"""``PredictiveLlm`` — the one-object API: train, generate, chat, serve, evaluate, learn online,
distill, remember, save and load.

Reference: PredictiveCoding.LLM/PredictiveLlm.cs:18-1114 and ChatSession.cs:15-55.  Method
names are the reference's in snake_case; options/results are the records of
``llm.options``.  Training runs the autograd ``DecoderLM`` on its device; for the dense
RMSNorm+RoPE family ``train_fused`` runs the same data through the sm_100a
``FusedDecoderTrainer`` (one GPU, or one rank per GPU under ``torchrun``).
"""
from __future__ import annotations

import math
import os
import struct
from typing import Callable, List, Optional, Sequence, Tuple

import torch

from ..io import checkpoint as ck
from ..models.config import DecoderLmConfig
from ..models.decoder_lm import DecoderLM
from ..optim.adam import Adam, LrSchedule
from . import distill as distill_mod
from .data import CorpusSource, StreamingTextDataset
from .eval import (ActivationProbe, BitsPerByteResult, PerplexityResult, TINY_EVAL_CORPUS, bits_per_byte, evaluate,
                   held_out, held_out_hashed, html_report, training_split, training_split_hashed)
from .generation import ChatTemplate, Sampler, self_speculative
from .memory import EpisodicMemory
from .options import (GenerationOptions, GenerationResult, OnlineLearnReport, TokenizerManifest, TokenOdometer,
                      TrainingOptions, TrainingReport)
from .pc_trainer import DEFAULT_ANCHOR_EVERY, PcDecoderTrainer
from .tokenizer import BpeTokenizer, ByteTokenizer, Tokenizer
from .trainer import step as train_step
from .trainer import step_parallel


class PredictiveLlm:
    def __init__(self, config: DecoderLmConfig, tokenizer: Optional[Tokenizer] = None, seed: int = 42,
                 device: Optional[str] = None):
        self.tokenizer = tokenizer or ByteTokenizer()
        if config.vocab != self.tokenizer.vocab_size:
            raise ValueError(f"Config vocab ({config.vocab}) must match the tokenizer ({self.tokenizer.vocab_size}).")
        self.seed = seed
        self.model = DecoderLM(config, seed=seed)
        if device is not None:
            self.model.to(device)
        self.odometer = TokenOdometer()
        self.memory: Optional[EpisodicMemory] = None
        self._online_opt: Optional[Adam] = None
        self._pc: Optional[PcDecoderTrainer] = None
        # iPC knobs (PredictiveLlm.cs:44-55)
        self.pc_anchor_every = DEFAULT_ANCHOR_EVERY
        self.pc_anchor_burst = 3
        self.pc_eta_state = 0.1
        self.pc_lr_weights = 0.3
        self.pc_clip_norm = 1.0
        self.pc_relax_steps = 1

    # ------------------------------------------------------------ factories
    @staticmethod
    def _config_2026(vocab, dim, blocks, heads, ff, max_seq) -> DecoderLmConfig:
        pattern = "".join("T" if b % 2 == 0 else "A" for b in range(blocks))
        return DecoderLmConfig(vocab, dim, blocks, heads, ff, max_seq, num_loops=2, loop_exit_tau=0.05,
                               mtp_weight=0.3, block_pattern=pattern, num_experts=4, moe_top_k=1, use_plan=True)

    @staticmethod
    def create_2026(dim=64, blocks=4, heads=4, ff_dim=128, max_seq=128, seed=42, tokenizer_corpus: str = None,
                    merges: int = 512) -> "PredictiveLlm":
        """Every mechanism on: pattern TATA, loops 2, MTP 0.3, 4 experts top-1, plan."""
        if tokenizer_corpus is not None:
            tok = BpeTokenizer()
            tok.train(tokenizer_corpus, merges)
        else:
            tok = ByteTokenizer()
        return PredictiveLlm(PredictiveLlm._config_2026(tok.vocab_size, dim, blocks, heads, ff_dim, max_seq), tok, seed)

    @staticmethod
    def create_small(tokenizer: Tokenizer, max_seq: int = 512, seed: int = 42) -> "PredictiveLlm":
        return PredictiveLlm(DecoderLmConfig.small(tokenizer.vocab_size, max_seq), tokenizer, seed)

    @staticmethod
    def create_base(tokenizer: Tokenizer, max_seq: int = 1024, seed: int = 42) -> "PredictiveLlm":
        return PredictiveLlm(DecoderLmConfig.base(tokenizer.vocab_size, max_seq), tokenizer, seed)

    @staticmethod
    def create_pc(dim=64, blocks=4, heads=4, ff_dim=256, max_seq=1024, seed=42) -> "PredictiveLlm":
        tok = ByteTokenizer()
        cfg = DecoderLmConfig(tok.vocab_size, dim, blocks, heads, ff_dim, max_seq, use_rms_norm=True, use_rope=True)
        return PredictiveLlm(cfg, tok, seed)

    # ------------------------------------------------------------ properties
    @property
    def config(self) -> DecoderLmConfig:
        return self.model.cfg

    @property
    def parameter_count(self) -> int:
        return self.model.parameter_count

    @property
    def active_parameter_count_per_token(self) -> int:
        return self.model.active_parameter_count_per_token

    @property
    def device(self):
        return self.model.wemb.device

    def to(self, device) -> "PredictiveLlm":
        self.model.to(device)
        return self

    # ------------------------------------------------------------ windows
    def _text_windows(self, text: str):
        seq = min(32, self.config.max_seq)
        ws = list(StreamingTextDataset(text.split("\n"), self.tokenizer, seq, max(1, seq // 2)).windows())
        return ws or [self._whole_text_window(text)]

    def _whole_text_window(self, text: str):
        ids = self.tokenizer.encode(text, add_bos=True, add_eos=True)
        n = min(len(ids), self.config.max_seq + 1)
        if n < 2:
            raise ValueError("Text too short to evaluate (needs at least 2 tokens).")
        return ids[: n - 1], ids[1:n]

    def _loss(self, t, y, training):
        return self.model.loss(t.view(1, -1), y.view(1, -1), -1, training)

    # ------------------------------------------------------------ training
    def train(self, corpus, options: Optional[TrainingOptions] = None) -> TrainingReport:
        """Train on a string (positional held-out split) or a CorpusSource (content-hashed split)."""
        opts = options or TrainingOptions()
        seq = min(opts.seq_len, self.config.max_seq)
        if isinstance(corpus, CorpusSource):
            data = StreamingTextDataset(corpus.lines, self.tokenizer, seq, opts.stride)
            return self._train_core(data, opts, True, None)
        data = StreamingTextDataset(corpus.split("\n"), self.tokenizer, seq, opts.stride)
        return self._train_core(data, opts, False, lambda: self._whole_text_window(corpus))

    def _train_core(self, data, opts: TrainingOptions, hashed: bool, fallback) -> TrainingReport:
        ws = list(data.windows())
        ev = list((held_out_hashed if hashed else held_out)(ws, opts.held_out_every))
        tr = list((training_split_hashed if hashed else training_split)(ws, opts.held_out_every))
        if opts.max_windows is not None and len(tr) > opts.max_windows:
            tr = tr[: opts.max_windows]
        if not tr:
            raise ValueError("Corpus too small: no training window. Shorten seq_len or feed more text.")
        if not ev:
            ev = [fallback() if fallback else tr[-1]]
        before = evaluate(self.model, ev)
        self.odometer.evaluated += before.tokens
        batches = [tr[i:i + opts.batch_windows] for i in range(0, len(tr), opts.batch_windows)]
        total = opts.epochs * len(batches)
        sched = LrSchedule(opts.peak_lr, opts.min_lr, max(1, total // 10), total)
        opt = opts.resume_optimizer or Adam()
        ps = list(self.model.parameters())
        if opts.checkpoint_every_steps > 0 and not opts.checkpoint_dir:
            raise ValueError("checkpoint_every_steps > 0 requires checkpoint_dir.")
        workers = max(1, min(opts.workers if opts.workers > 0 else (os.cpu_count() or 1), opts.batch_windows))
        replicas = None
        if workers > 1:
            models = [self.model] + [DecoderLM(self.config, seed=self.seed + w).to(self.device) for w in range(1, workers)]
            replicas = ([list(m.parameters()) for m in models],
                        [(lambda mm: (lambda t, y, trn: mm.loss(t.view(1, -1), y.view(1, -1), -1, trn)))(m)
                         for m in models])
        best_ppl, best_dir = float("inf"), None
        first = last = 0.0
        step = 0
        for epoch in range(opts.epochs):
            esum = 0.0
            for batch in batches:
                lr = sched.at(step)
                if replicas:
                    last = step_parallel(replicas[0], replicas[1], batch, opt, lr, opts.clip_norm)
                else:
                    last = train_step(ps, batch, self._loss, opt, lr, opts.clip_norm)
                if step == 0:
                    first = last
                esum += last
                step += 1
                if opts.checkpoint_every_steps > 0 and step % opts.checkpoint_every_steps == 0:
                    ppl = evaluate(self.model, ev).perplexity
                    if not opts.keep_best_by_perplexity or ppl < best_ppl:
                        best_ppl, best_dir = ppl, opts.checkpoint_dir
                        self.save_resumable(best_dir, opt, opts.checkpoint_precision)
            if opts.on_epoch_end:
                opts.on_epoch_end(epoch + 1, esum / len(batches))
        after = evaluate(self.model, ev)
        self.odometer.evaluated += after.tokens
        self.odometer.trained += sum(len(t) for t, _ in tr) * opts.epochs
        return TrainingReport(before.perplexity, after.perplexity, first, last, step, len(tr), len(ev),
                              best_ppl if best_dir else float("nan"), best_dir)

    def train_fused(self, corpus: str, batch: int, steps: int, lr: float = 3e-4, weight_decay: float = 0.1,
                    process_group=None, device: Optional[str] = None):
        """Train on the sm_100a fused trainer (dense RMSNorm+RoPE configs); weights come back into
        ``self.model``.  Returns the per-step losses."""
        from ..engine.fused_trainer import FusedDecoderTrainer
        seq = self.config.max_seq
        ws = list(StreamingTextDataset(corpus.split("\n"), self.tokenizer, seq, seq).windows())
        if len(ws) < batch:
            raise ValueError(f"need at least {batch} windows of {seq} tokens")
        dev = device or "cuda"
        trn = FusedDecoderTrainer(self.config, batch, seq, device=dev, lr=lr, weight_decay=weight_decay,
                                  model=self.model.cpu(), process_group=process_group, use_graph=False)
        losses = []
        for s in range(steps):
            idx = [(s * batch + i) % len(ws) for i in range(batch)]
            tok = torch.tensor([ws[i][0] for i in idx])
            tgt = torch.tensor([ws[i][1] for i in idx])
            losses.append(trn.step(tok, tgt))
            self.odometer.trained += batch * seq
        trn.export_model(self.model)
        return losses

    # ------------------------------------------------------------ memory
    @torch.no_grad()
    def embed(self, text: str) -> torch.Tensor:
        ids = self.tokenizer.encode(text, add_bos=True) or [self.tokenizer.bos]
        ids = ids[: self.config.max_seq]
        h = self.model.hidden(torch.tensor(ids, device=self.device))
        start = 1 if h.shape[0] > 1 else 0
        return h[start:].mean(0).float().cpu()

    def remember(self, text: str) -> None:
        if self.memory is None:
            self.memory = EpisodicMemory(self.config.dim)
        self.memory.remember(self.embed(text), text)

    def _prepend_recalled(self, prompt: str, top_k: int) -> str:
        hits = self.memory.recall(self.embed(prompt), top_k)
        kept = []
        for text, _ in hits:
            cand = "\n".join(kept + [text]) + "\n" + prompt
            if len(self.tokenizer.encode(cand, add_bos=True)) < self.config.max_seq:
                kept.append(text)
            else:
                break
        return prompt if not kept else "\n".join(kept) + "\n" + prompt

    # ------------------------------------------------------------ generation
    def generate(self, prompt: str, max_new_tokens: int = 64, options: Optional[GenerationOptions] = None) -> str:
        return self.generate_detailed(prompt, max_new_tokens, options).text

    @staticmethod
    def _cut_at_stop(text: str, stops) -> Tuple[str, bool]:
        if not stops:
            return text, False
        cut = -1
        for s in stops:
            if s:
                i = text.find(s)
                if i >= 0 and (cut < 0 or i < cut):
                    cut = i
        return (text, False) if cut < 0 else (text[:cut], True)

    def generate_detailed(self, prompt: str, max_new_tokens: int = 64,
                          options: Optional[GenerationOptions] = None) -> GenerationResult:
        o = options or GenerationOptions()
        if o.use_memory and self.memory is not None and self.memory.count > 0:
            prompt = self._prepend_recalled(prompt, o.memory_top_k)
        ctx = self.tokenizer.encode(prompt, add_bos=True)
        if len(ctx) >= self.config.max_seq:
            raise ValueError(f"Prompt is {len(ctx)} tokens; the window holds {self.config.max_seq}.")
        if o.learn_from_prompt and len(ctx) >= 2:
            self.learn(prompt)
        saved_plan = None
        if o.settle_plan_steps > 0 and self.config.use_plan and len(ctx) >= 2:
            saved_plan = self.model.plan.detach().clone()
            self.model.settle_plan(torch.tensor(ctx, device=self.device), o.settle_plan_steps, o.settle_plan_lr)
        try:
            if o.sampling is not None:
                return self._sample_loop(ctx, max_new_tokens, o)
            eos = self.tokenizer.eos if o.stop_at_eos else -1
            run = self_speculative(self.model, ctx, max_new_tokens, eos)
            gen = run.tokens[len(ctx):]
            text, _ = self._cut_at_stop(self.tokenizer.decode(gen), o.stop_sequences)
            self.odometer.prompted += len(ctx)
            self.odometer.generated += len(gen)
            return GenerationResult(text, run.forwards, run.drafted, run.accepted)
        finally:
            if saved_plan is not None:
                with torch.no_grad():
                    self.model.plan.copy_(saved_plan)

    @torch.no_grad()
    def _sample_loop(self, ctx, max_new, o: GenerationOptions) -> GenerationResult:
        so = o.sampling
        sampler = Sampler(so.seed if so.seed is not None else 42)
        seq, gen, forwards, text = list(ctx), [], 0, ""
        while len(gen) < max_new and len(seq) < self.config.max_seq:
            logits = self.model.forward(torch.tensor(seq, device=self.device))
            forwards += 1
            nxt = sampler.sample(logits[-1], seq, so)
            if o.stop_at_eos and nxt == self.tokenizer.eos:
                break
            gen.append(nxt)
            seq.append(nxt)
            text, cut = self._cut_at_stop(self.tokenizer.decode(gen), o.stop_sequences)
            if cut:
                break
        self.odometer.prompted += len(ctx)
        self.odometer.generated += len(gen)
        return GenerationResult(text, forwards, 0, 0)

    def create_server(self, device=None):
        from .serving import LlmServer, export
        return LlmServer(export(self.model, device or self.device), self.tokenizer)

    def start_chat(self, system: Optional[str] = None) -> "ChatSession":
        return ChatSession(self, system)

    # ------------------------------------------------------------ evaluation
    def evaluate(self, text: str, max_windows: Optional[int] = None) -> PerplexityResult:
        r = evaluate(self.model, self._text_windows(text), max_windows=max_windows)
        self.odometer.evaluated += r.tokens
        return r

    def evaluate_bits_per_byte(self, text: str) -> BitsPerByteResult:
        r = bits_per_byte(self.model, self.tokenizer, text, self.config.max_seq,
                          fallback_window=self._whole_text_window(text))
        self.odometer.evaluated += r.tokens
        return r

    # ------------------------------------------------------------ online learning
    def _mean_loss(self, ws) -> float:
        with torch.no_grad():
            return sum(float(self._loss(torch.tensor(t, device=self.device), torch.tensor(y, device=self.device), False))
                       for t, y in ws) / len(ws)

    def learn(self, text: str, steps: int = 1, learning_rate: float = 1e-3) -> OnlineLearnReport:
        if steps < 1:
            raise ValueError("steps must be >= 1.")
        ws = self._text_windows(text)
        self._online_opt = self._online_opt or Adam()
        ntok = sum(len(t) for t, _ in ws)
        self.odometer.absorbed += ntok * steps
        self.odometer.evaluated += ntok * 2
        before = self._mean_loss(ws)
        ps = list(self.model.parameters())
        for _ in range(steps):
            train_step(ps, ws, self._loss, self._online_opt, learning_rate, 1.0)
        return OnlineLearnReport(before, self._mean_loss(ws), steps)

    def learn_pc(self, text: str, steps: int = 1, count_as_training: bool = False,
                 measure_surprise: bool = True) -> OnlineLearnReport:
        if steps < 1:
            raise ValueError("steps must be >= 1.")
        if self._pc is None:
            self._pc = PcDecoderTrainer(self.model, self.pc_relax_steps, self.pc_eta_state, self.pc_lr_weights,
                                        self.pc_clip_norm, self.pc_anchor_every, self.pc_anchor_burst)
        ws = self._text_windows(text)
        ntok = sum(len(t) for t, _ in ws)
        if count_as_training:
            self.odometer.trained += ntok * steps
        else:
            self.odometer.absorbed += ntok * steps
        if measure_surprise:
            self.odometer.evaluated += ntok * 2
        before = self._mean_loss(ws) if measure_surprise else 0.0
        for _ in range(steps):
            for t, y in ws:
                self._pc.step(t, y)
        after = self._mean_loss(ws) if measure_surprise else 0.0
        return OnlineLearnReport(before, after, steps)

    def distill_from(self, teacher: Callable[[str], str], prompts: Sequence[str], steps: int = 20,
                     learning_rate: float = 0.01, cache_dir: Optional[str] = None) -> float:
        data = distill_mod.build_dataset(prompts, teacher, cache_dir)
        opt = Adam()
        loss = 0.0
        for _ in range(steps):
            loss = distill_mod.step(self.model, self.tokenizer, data, opt, learning_rate)
        return loss

    def distill_on_policy(self, teacher_correct: Callable[[str, str], str], prompts: Sequence[str],
                          learning_rate: float = 0.01, draft_tokens: int = 16) -> float:
        return distill_mod.on_policy_round(self.model, self.tokenizer, prompts, teacher_correct, Adam(),
                                           learning_rate, draft_tokens)

    # ------------------------------------------------------------ persistence
    def weights_are_finite(self) -> bool:
        return all(bool(torch.isfinite(p).all()) for p in self.model.parameters())

    def save(self, directory: str, precision: str = "float32") -> None:
        """Config, weights, tokenizer, odometer, memory and online-Adam moments in one keyed store."""
        os.makedirs(directory, exist_ok=True)
        ps = self.model.reference_parameters()
        cfg_json = self.config.to_json().encode()
        kind = "bpe" if isinstance(self.tokenizer, BpeTokenizer) else (
            "byte" if isinstance(self.tokenizer, ByteTokenizer) else type(self.tokenizer).__name__)
        manifest = TokenizerManifest(kind, self.tokenizer.vocab_size, "").to_json()
        odo = self.odometer.to_json()
        mem = self.memory.live_entries_oldest_first() if self.memory is not None else None
        max_len = max(max(9 + (p.numel() * (4 if precision == "float32" else 2)) for p in ps),
                      len(cfg_json), len(manifest), len(odo))
        bits = ck.page_size_bits_for(max_len)
        ck.clear_store(directory)
        ck.write_page_size_hint(directory, bits)
        with ck.CheckpointStore(directory, bits, recover=False) as st:
            st.put_blob(ck.VERSION_KEY, struct.pack("<i", ck.FORMAT_VERSION))
            st.put_blob(ck.CONFIG_KEY, cfg_json)
            st.put_blob(ck.TOKENIZER_MANIFEST_KEY, manifest)
            if isinstance(self.tokenizer, BpeTokenizer):
                merges = self.tokenizer.merges_in_rank_order()
                st.put_blob(ck.TOKENIZER_HEADER_KEY, struct.pack("<Bii", 1 if self.tokenizer.word_split else 0,
                                                                 self.tokenizer.vocab_size, len(merges)))
                for m, (a, b, i) in enumerate(merges):
                    st.put_blob(ck.MERGE_BASE + m, struct.pack("<iii", a, b, i))
            for i, p in enumerate(ps):
                st.upsert_tensor(i, p, precision)
            st.put_blob(ck.ODOMETER_KEY, odo)
            if mem is not None:
                st.put_blob(ck.MEMORY_HEADER_KEY, struct.pack("<iii", self.memory.key_dim, self.memory.capacity, len(mem)))
                for i, (k, text) in enumerate(mem):
                    tb = text.encode("utf-8")
                    st.put_blob(ck.MEMORY_ENTRY_BASE + i, k.numpy().astype("<f4").tobytes() + struct.pack("<i", len(tb)) + tb)
            if self._online_opt is not None:
                st.put_blob(ck.OPTIMIZER_STEP_KEY, struct.pack("<i", self._online_opt.step_count))
                for i, p in enumerate(self.model.parameters()):
                    mv = self._online_opt.moments_for(p)
                    m = mv[0] if mv else torch.zeros_like(p)
                    v = mv[1] if mv else torch.zeros_like(p)
                    st.put_blob(ck.MOMENT_M_BASE + i, m.detach().float().cpu().numpy().astype("<f4").tobytes())
                    st.put_blob(ck.MOMENT_V_BASE + i, v.detach().float().cpu().numpy().astype("<f4").tobytes())
            st.commit()

    @staticmethod
    def load(directory: str, tokenizer: Optional[Tokenizer] = None, seed: int = 42,
             restore_optimizer: bool = True) -> "PredictiveLlm":
        bits = ck.read_page_size_hint(directory)
        with ck.CheckpointStore(directory, bits, recover=True) as st:
            v = st.get_blob(ck.VERSION_KEY)
            if v is None or len(v) < 4 or struct.unpack("<i", v[:4])[0] != ck.FORMAT_VERSION:
                raise ValueError(f"'{directory}' is not a v{ck.FORMAT_VERSION} LLM checkpoint.")
            cfg_b = st.get_blob(ck.CONFIG_KEY)
            if cfg_b is None:
                raise ValueError(f"Checkpoint under '{directory}' is missing its config.")
            cfg = DecoderLmConfig.from_json(cfg_b.decode())
            man = TokenizerManifest.from_json(st.get_blob(ck.TOKENIZER_MANIFEST_KEY))
            if man.kind == "byte":
                tokenizer = tokenizer or ByteTokenizer()
            elif man.kind == "bpe":
                if tokenizer is not None:
                    raise ValueError("This model carries its own BPE tokenizer — do not pass one to load.")
                ws, vocab, count = struct.unpack("<Bii", st.get_blob(ck.TOKENIZER_HEADER_KEY))
                merges = [struct.unpack("<iii", st.get_blob(ck.MERGE_BASE + m)) for m in range(count)]
                tokenizer = BpeTokenizer.from_merges(bool(ws), vocab, merges)
            elif tokenizer is None:
                raise ValueError(f"This model was saved with a custom tokenizer ({man.kind}) — pass it to load.")
            if tokenizer.vocab_size != man.vocab_size:
                raise ValueError("Tokenizer vocab size does not match the saved model.")
            llm = PredictiveLlm(cfg, tokenizer, seed)
            ps = llm.model.reference_parameters()
            tensors = []
            for i in range(len(ps)):
                b = st.get_blob(i)
                if b is None:
                    raise ValueError(f"Checkpoint under '{directory}' is missing tensor {i}.")
                a, _ = ck.read_tensor_blob(b)
                if a.size != ps[i].numel():
                    raise ValueError(f"Shape mismatch for tensor {i}.")
                tensors.append(a)
            if st.get_blob(len(ps)) is not None:
                raise ValueError(f"Checkpoint under '{directory}' has more tensors than the model ({len(ps)}).")
            llm.model.load_reference_parameters(tensors)
            odo = st.get_blob(ck.ODOMETER_KEY)
            if odo is not None:
                llm.odometer.load_json(odo)
            mh = st.get_blob(ck.MEMORY_HEADER_KEY)
            if mh is not None:
                kd, cap, cnt = struct.unpack("<iii", mh)
                if kd != cfg.dim:
                    raise ValueError(f"Memory key dim {kd} != model embedding dim {cfg.dim}.")
                mem = EpisodicMemory(kd, cap)
                for i in range(cnt):
                    e = st.get_blob(ck.MEMORY_ENTRY_BASE + i)
                    key = torch.frombuffer(bytearray(e[:4 * kd]), dtype=torch.float32).clone()
                    n = struct.unpack_from("<i", e, 4 * kd)[0]
                    mem.remember(key, e[4 * kd + 4:4 * kd + 4 + n].decode("utf-8"))
                llm.memory = mem
            sb = st.get_blob(ck.OPTIMIZER_STEP_KEY) if restore_optimizer else None
            if sb is not None:
                opt = Adam()
                for i, p in enumerate(llm.model.parameters()):
                    m = torch.frombuffer(bytearray(st.get_blob(ck.MOMENT_M_BASE + i)), dtype=torch.float32).view_as(p)
                    vv = torch.frombuffer(bytearray(st.get_blob(ck.MOMENT_V_BASE + i)), dtype=torch.float32).view_as(p)
                    opt.set_moments(p, m, vv)
                opt.restore_step_count(struct.unpack("<i", sb)[0])
                llm._online_opt = opt
        return llm

    def save_resumable(self, directory: str, optimizer: Adam, precision: str = "float32") -> None:
        self.save(directory, precision)
        ps = list(self.model.parameters())
        ck.save_opt1(os.path.join(directory, "optimizer.bin"), ps, optimizer.step_count,
                     [optimizer.moments_for(p) for p in ps])

    @staticmethod
    def load_with_optimizer(directory: str, tokenizer: Optional[Tokenizer] = None, seed: int = 42):
        llm = PredictiveLlm.load(directory, tokenizer, seed)
        opt = Adam()
        path = os.path.join(directory, "optimizer.bin")
        if os.path.exists(path):
            ps = list(llm.model.parameters())
            t, mv = ck.load_opt1(path, ps)
            for p, (m, v) in zip(ps, mv):
                opt.set_moments(p, m, v)
            opt.restore_step_count(t)
        return llm, opt

    def report(self, path: str, eval_text: Optional[str] = None) -> str:
        text = eval_text or TINY_EVAL_CORPUS
        probe = ActivationProbe()
        ids = self.tokenizer.encode(text.split("\n")[0], add_bos=True)[: self.config.max_seq]
        with torch.no_grad():
            self.model.forward(torch.tensor(ids, device=self.device), False, probe)
        return html_report(path, "PredictiveLlm yardstick", self.evaluate(text), probe,
                           {"parameters": self.parameter_count, "odometer": str(self.odometer)})


class ChatSession:
    """Multi-turn chat over the chat template (ChatSession.cs:15-55)."""

    def __init__(self, llm: PredictiveLlm, system: Optional[str] = None):
        self.llm, self.system = llm, system
        self.turns: List[Tuple[str, str]] = []

    def say(self, user: str, max_new_tokens: int = 64, options: Optional[GenerationOptions] = None) -> str:
        self.turns.append(("user", user))
        prompt = ChatTemplate.format(self.system, self.turns)
        # keep the most recent turns that fit the window
        while len(self.llm.tokenizer.encode(prompt, add_bos=True)) >= self.llm.config.max_seq and len(self.turns) > 1:
            self.turns.pop(0)
            prompt = ChatTemplate.format(self.system, self.turns)
        o = options or GenerationOptions(stop_sequences=["<|"])
        reply = self.llm.generate(prompt, max_new_tokens, o).strip()
        self.turns.append(("assistant", reply))
        return reply

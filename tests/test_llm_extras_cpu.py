"""GPT family, tiny LM, quantisation, GEMM routing, memory budget, continual learning,
translation and summarisation on the CPU."""
import math
import os
import tempfile

import pytest
import torch

from predicitivecoding_b200.llm.gpt import GptModel, ModernPresets, TransformerConfig
from predicitivecoding_b200.llm.tiny import TinyTransformerLM, sgd_step
from predicitivecoding_b200.llm import quant
from predicitivecoding_b200.llm.gemm_provider import Gemm, GemmMatMul, TorchGemmProvider
from predicitivecoding_b200.llm.memory_budget import measure
from predicitivecoding_b200.llm.continual import ContinualLearner, ContinualOptions
from predicitivecoding_b200.llm import translation as tr
from predicitivecoding_b200.llm.summarize import ExtractiveSummarizer, SummaryOptions, split_sentences
from predicitivecoding_b200.llm.facade import PredictiveLlm
from predicitivecoding_b200.models.config import DecoderLmConfig
from predicitivecoding_b200.models.decoder_lm import DecoderLM

BASE = dict(vocab_size=50, embed_dim=32, num_heads=4, num_layers=2, feed_forward_dim=64)
CONFIGS = [
    TransformerConfig(**BASE),
    TransformerConfig(**BASE, positional="alibi", num_experts=3, moe_top_k=2),
    TransformerConfig(**BASE, positional="rotary", window_size=4, num_sink_tokens=2),
    TransformerConfig(**BASE, positional="rotary", use_qk_norm=True, attn_logit_softcap=5.0, final_logit_softcap=3.0,
                      num_kv_heads=1, kv_cache_half=False),
    ModernPresets.llama3_style(vocab=50, embed=32, heads=4, kv_heads=2, layers=2, ff=64),
    ModernPresets.nemotron_style(vocab=50, embed=32, heads=4, layers=4, ff=64),
    ModernPresets.deepseek_style(vocab=50, embed=32, heads=4, layers=2, ff=64),
]


@pytest.mark.parametrize("cfg", CONFIGS, ids=lambda c: f"{c.attention}-{c.positional}-{c.block_pattern}-{c.window_size}")
def test_gpt_incremental_decode_equals_full_forward(cfg):
    m = GptModel(cfg, seed=1).eval()
    toks = torch.randint(0, 50, (2, 12), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        full = m(toks)
        cache = m.create_cache()
        pre = m(toks[:, :5], cache, 0)
        steps = [m.step(toks[:, t], t, cache) for t in range(5, 12)]
    inc = torch.cat([pre, torch.stack(steps, 1)], 1)
    assert torch.allclose(full, inc, atol=1e-5)
    if cfg.window_size:
        assert cache.layers[0].length == cfg.num_sink_tokens + cfg.window_size
    assert cache.bytes_used > 0 and m.forward_tokens == 24 + 5 * 2 + 7 * 2


def test_gpt_config_validation_and_json():
    with pytest.raises(ValueError):
        TransformerConfig(embed_dim=30, num_heads=4).validate()
    with pytest.raises(ValueError):
        TransformerConfig(num_sink_tokens=2).validate()
    with pytest.raises(ValueError):
        TransformerConfig(num_layers=2, block_pattern="AX").validate()
    c = ModernPresets.deepseek_style()
    assert TransformerConfig.from_json(c.to_json()) == c and c.rope_head_dim % 2 == 0
    assert ModernPresets.nemotron_style(layers=8).block_pattern == "TTTATTTA"


def test_gpt_kv_half_cache_and_generate():
    cfg = TransformerConfig(**BASE, kv_cache_half=True, positional="rotary")
    m = GptModel(cfg, seed=2).eval()
    c = m.create_cache()
    m(torch.tensor([[1, 2, 3]]), c, 0)
    assert c.layers[0].k.dtype == torch.float16 and c.bytes_used == 2 * 3 * 4 * 8 * 2 * 2
    out = m.generate([1, 2, 3], 5)
    assert len(out) == 8


def test_tiny_transformer_sgd_learns():
    m = TinyTransformerLM(12, 16, 32, seed=0)
    toks, tgts = [1, 2, 3, 4, 5, 6], [2, 3, 4, 5, 6, 7]
    l0 = float(m.loss(toks, tgts).detach())
    for _ in range(200):
        for p in m.parameters():
            p.grad = None
        m.loss(toks, tgts, True).backward()
        sgd_step(m.parameters(), 0.5)
    assert float(m.loss(toks, tgts).detach()) < 0.5 * l0


def test_bf16_rne_and_nan():
    x = torch.tensor([1.0, 1.00390625, 1.01171875, float("nan"), -2.5])
    bits = quant.bf16_bits(x)
    assert bits[0] == 0x3F80 and bits[1] == 0x3F80 and bits[2] == 0x3F82     # ties to even
    assert torch.isnan(quant.bf16_from_bits(bits[3:4]))[0]
    assert torch.equal(quant.bf16_from_bits(bits), x.to(torch.bfloat16).float()) is False  # NaN != NaN
    assert torch.equal(quant.bf16_from_bits(bits)[[0, 1, 2, 4]], x[[0, 1, 2, 4]].to(torch.bfloat16).float())


def test_low_precision_and_int_quantisation():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(16, 33, generator=g)
    x = torch.randn(33, generator=g)
    ref = w @ x
    for m, tol in [(quant.LowPrecisionMatrix(w, "bf16"), 0.02), (quant.LowPrecisionMatrix(w, "fp16"), 0.002),
                   (quant.Int8Matrix(w), 0.02), (quant.Int4Matrix(w), 0.25)]:
        assert (m.matvec(x) - ref).abs().max() <= tol * ref.abs().max()
    q4 = quant.Int4Matrix(w)
    assert q4.packed.shape == (16, 17) and q4.memory_bytes == 16 * 17 + 16 * 4
    assert q4.unpack().abs().max() <= 7
    one = quant.Int4Matrix(torch.tensor([[-7.0, 7.0, 1.0]]))
    assert int(one.packed[0, 0]) == ((7 << 4) | 9) and int(one.packed[0, 1]) == 1
    q8 = quant.Int8Matrix(w)
    assert q8.q.dtype == torch.int8 and q8.q.abs().max() == 127


def test_gemm_provider_routes_and_autograd():
    Gemm.set_provider(TorchGemmProvider())
    Gemm.calls.clear()
    a = torch.randn(4, 5, requires_grad=True)
    b = torch.randn(5, 3, requires_grad=True)
    y = GemmMatMul.apply(a, b)
    y.sum().backward()
    assert torch.allclose(y, a @ b) and Gemm.calls["torch"] == 3
    assert torch.allclose(a.grad, torch.ones(4, 3) @ b.T)
    mixed = Gemm.matmul_mixed(a.detach(), b.detach())
    assert torch.allclose(mixed, a.detach() @ b.detach(), atol=1e-2)
    with pytest.raises(ValueError):
        Gemm.matmul(torch.randn(2, 3), torch.randn(4, 2))


def test_memory_budget():
    r = measure(DecoderLmConfig(64, 32, 2, 2, 64, 32), 16)
    assert r.gradient_bytes == r.parameter_bytes and r.adam_state_bytes == 2 * r.parameter_bytes
    assert r.activation_bytes > 0 and r.total_bytes > 4 * r.parameter_bytes
    assert r.project_fp16_bytes < r.total_bytes and "fp16 projection" in r.describe()
    with pytest.raises(ValueError):
        measure(DecoderLmConfig(64, 32, 2, 2, 64, 32), 64)


def test_continual_learner_absorbs_and_guards():
    llm = PredictiveLlm.create_pc(dim=32, blocks=1, heads=2, ff_dim=64, max_seq=64)
    drifts = []
    cl = ContinualLearner(llm, ContinualOptions(seq_len=16, stride=8, base_lr=0.01, steps=3, guardrail_every=1,
                                                drift_threshold=-1.0), yardstick_text="the sky is blue today.")
    cl.on_drift = drifts.append
    s1 = cl.absorb("the cat sat on the mat and the cat sat again.")
    assert s1.surprise_after < s1.surprise_before and cl.replay_size > 0
    s2 = cl.absorb("a dog ran in the park.")
    assert s2.replay_windows > 0 and cl.absorb_count == 2 and len(drifts) == 2
    assert math.isfinite(cl.baseline_perplexity)


def test_translation_examples_and_roundtrip():
    pairs = [tr.SentencePair("hello", "ciao", "it"), tr.SentencePair("cat", "gatto", "it")]
    tok = tr.train_tokenizer(pairs, 20)
    toks, tgts = tr.build_example(tok, "hello", "ciao", "it")
    p = tok.encode(tr.prompt_text("hello", "it"))
    assert toks[0] == tok.bos and tgts[:len(p)] == [-1] * len(p) and tgts[-1] == tok.eos
    assert tr.build_prompt(tok, "cat", "it")[0] == tok.bos
    assert len(tr.build_examples(pairs, tok, 4)) == 0 and len(tr.build_examples(pairs, tok, 256)) == 2
    model = DecoderLM(DecoderLmConfig(tok.vocab_size, 16, 1, 2, 32, 64), seed=0)
    t = tr.Translator(model, tok)
    with tempfile.TemporaryDirectory() as d:
        t.save(d)
        back = tr.Translator.load(d)
        for a, b in zip(model.parameters(), back.model.parameters()):
            assert torch.equal(a, b)
        assert back.translate("cat", "it", 5) == t.translate("cat", "it", 5)


def test_translation_tsv_reader(tmp_path):
    f = tmp_path / "c.tsv"
    f.write_text("# comment\nit\thello\tciao\n\nbad line\nfr\tcat\tchat\n")
    got = list(tr.read_tsv(str(f)))
    assert [(p.target_tag, p.source, p.target) for p in got] == [("it", "hello", "ciao"), ("fr", "cat", "chat")]


def test_sentence_split_rules():
    s = split_sentences("Dr. Smith paid 3.5 dollars. He left! J. Doe stayed? yes it was fine")
    assert s == ["Dr. Smith paid 3.5 dollars.", "He left!", "J. Doe stayed? yes it was fine"]


@pytest.mark.parametrize("method", ["centroid", "textrank", "termfrequency"])
def test_summarizer_methods(method):
    text = ("Cats are small furry animals. Cats like to sleep all day. Dogs bark at cats. "
            "The stock market fell today. Cats and dogs are common pets.")
    out = ExtractiveSummarizer().summarize(text, SummaryOptions(max_sentences=2, ratio=1.0, method=method,
                                                                language="en"))
    sents = split_sentences(out)
    assert len(sents) == 2 and all(x in text for x in sents)
    assert text.index(sents[0]) < text.index(sents[1])           # reading order
    assert "stock market" not in out
    assert ExtractiveSummarizer().summarize("One sentence only") == "One sentence only"


def test_device_pretrainer_cpu_path(tmp_path):
    from predicitivecoding_b200.engine.pretrainer import DevicePretrainOptions, lr_at, pretrain
    from predicitivecoding_b200.llm.data import CorpusSource
    llm = PredictiveLlm.create_pc(dim=32, blocks=1, heads=2, ff_dim=64, max_seq=64)
    text = "\n".join(f"line {i} the cat sat on the mat and looked at the dog {i % 7}." for i in range(60))
    seen = []
    o = DevicePretrainOptions(seq_len=16, stride=16, micro_batch_windows=2, peak_lr=3e-3, min_lr=3e-4,
                              warmup_steps=2, max_steps=12, eval_every_steps=4, eval_windows=4, held_out_every=5,
                              quality_every_steps=6, sample_tokens=4, checkpoint_dir=str(tmp_path / "ck"),
                              checkpoint_every_steps=6, log_path=str(tmp_path / "log.jsonl"),
                              on_progress=seen.append)
    rep = pretrain(llm, CorpusSource.from_text(text), o)
    assert rep.steps == 12 and rep.tokens == 12 * 2 * 16 and len(seen) == 12
    assert math.isfinite(rep.final_eval_loss) and rep.best_eval_loss <= rep.final_eval_loss + 1.0
    assert seen[5].sample is not None and seen[5].bits_per_byte is not None
    assert len(open(tmp_path / "log.jsonl").read().splitlines()) == 12
    assert os.path.isdir(tmp_path / "ck" / "best")
    assert lr_at(1, 100, o) == pytest.approx(1.5e-3) and lr_at(100, 100, o) == pytest.approx(3e-4)

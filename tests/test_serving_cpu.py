"""Exporter to the step-by-step KV-cache model, the text / batched generators and the token-loss
evaluator (Serving/GptExporter.cs, Generation/TextGenerator.cs, BatchedGenerator.cs,
Training/CrossEntropy.cs)."""
import math

import pytest
import torch

from predicitivecoding_b200.llm.eval import evaluate_gpt, token_loss
from predicitivecoding_b200.llm.generation import BatchedGenerator, SamplingOptions, TextGenerator
from predicitivecoding_b200.llm.serving import InferenceModel, StepModelServer, export, export_gpt
from predicitivecoding_b200.llm.tokenizer import ByteTokenizer
from predicitivecoding_b200.models.config import DecoderLmConfig
from predicitivecoding_b200.models.decoder_lm import DecoderLM

CFGS = {
    "temporal+plan+mtp": dict(block_pattern="TATA", use_plan=True, mtp_weight=0.3, num_blocks=4),
    "moe": dict(num_experts=4, moe_top_k=2),
    "rms+rope+swiglu": dict(use_rms_norm=True, use_rope=True, ffn="swiglu"),
}


def _model(kind, seed=3):
    kw = dict(vocab=260, dim=64, num_blocks=2, num_heads=4, ff_dim=128, max_seq=48)
    kw.update(CFGS[kind])
    m = DecoderLM(DecoderLmConfig(**kw), seed=seed).eval()
    with torch.no_grad():
        if m.plan is not None:
            m.plan.normal_(0, 0.1)
    return m


@pytest.mark.parametrize("kind", list(CFGS))
def test_exported_step_model_matches_the_trained_forward(kind):
    m = _model(kind)
    g = export_gpt(m).eval()
    tok = torch.randint(0, 260, (1, 30), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = m(tok)[0]
        cache = g.create_cache()
        got = torch.stack([g.step(int(t), i, cache).reshape(-1) for i, t in enumerate(tok[0])])
    assert float((ref - got).abs().max()) < 1e-4


def test_export_refuses_loops_and_dispatches_on_block_family():
    looped = DecoderLM(DecoderLmConfig(vocab=260, dim=64, num_blocks=2, num_heads=4, ff_dim=128, max_seq=48,
                                       num_loops=2))
    with pytest.raises(NotImplementedError):
        export_gpt(looped)
    assert isinstance(export(_model("temporal+plan+mtp")), StepModelServer)
    assert isinstance(export(_model("moe")), InferenceModel)


def test_plan_folds_into_the_batched_inference_model():
    m = DecoderLM(DecoderLmConfig(vocab=260, dim=64, num_blocks=2, num_heads=4, ff_dim=128, max_seq=48,
                                  use_plan=True), seed=5).eval()
    with torch.no_grad():
        m.plan.normal_(0, 0.2)
    inf = InferenceModel(m, device="cpu", dtype=torch.float32)
    tok = torch.randint(0, 260, (2, 12), generator=torch.Generator().manual_seed(2))
    cache = inf.new_cache(2)
    with torch.no_grad():
        assert torch.allclose(inf.prefill(tok, cache), m(tok), atol=1e-4)


def test_text_generator_matches_greedy_steps_and_stops_at_eos():
    tok = ByteTokenizer()
    g = export_gpt(_model("rms+rope+swiglu")).eval()
    opts = SamplingOptions(greedy=True, max_new_tokens=10)
    seen = []
    out = TextGenerator(g, tok).generate_tokens(tok.encode("hi", add_bos=True), opts, on_token=seen.append)
    assert out == seen and len(out) <= 10
    # the same tokens by hand
    cache, ids, pos = g.create_cache(), tok.encode("hi", add_bos=True), 0
    for t in ids:
        logits = g.step(t, pos, cache)
        pos += 1
    ref = []
    for _ in range(10):
        nxt = int(torch.argmax(logits.reshape(-1)))
        if nxt == tok.eos:
            break
        ref.append(nxt)
        logits = g.step(nxt, pos, cache)
        pos += 1
    assert out == ref
    # context limit: a prompt that fills the window generates nothing
    full = [tok.bos] + [65] * (g.max_seq_len - 1)
    assert TextGenerator(g, tok).generate_tokens(full, opts) == []


def test_batched_generator_equals_independent_text_generators():
    tok = ByteTokenizer()
    g = export_gpt(_model("moe")).eval()
    prompts = ["ab", "hello", ""]
    opts = SamplingOptions(temperature=0.8, top_k=20, max_new_tokens=8, seed=11)
    batched = BatchedGenerator(g, tok).generate_batch([tok.encode(p, add_bos=True) for p in prompts], opts)
    for i, p in enumerate(prompts):
        o = SamplingOptions(temperature=0.8, top_k=20, max_new_tokens=8, seed=11 + i)
        assert batched[i] == TextGenerator(g, tok).generate_tokens(tok.encode(p, add_bos=True), o)
    assert len(BatchedGenerator(g, tok).generate(prompts, opts)) == 3


def test_token_loss_and_teacher_forced_evaluation():
    logits = torch.tensor([1.0, 2.0, 3.0])
    assert abs(token_loss(logits, 2) - (math.log(math.exp(1) + math.exp(2) + math.exp(3)) - 3)) < 1e-9
    g = export_gpt(_model("rms+rope+swiglu")).eval()
    toks = list(range(65, 85))
    loss, ppl = evaluate_gpt(g, toks)
    with torch.no_grad():
        lg = g(torch.tensor([toks[:-1]]))[0]
    ref = float(torch.nn.functional.cross_entropy(lg.double(), torch.tensor(toks[1:])))
    assert abs(loss - ref) < 1e-4 and abs(ppl - math.exp(loss)) < 1e-9
    assert evaluate_gpt(g, [5]) == (0.0, 1.0)

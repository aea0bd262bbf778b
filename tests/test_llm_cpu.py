"""LLM stack on the CPU: tokenizers, data, evaluation, generation, serving, facade, formats."""
import math
import os
import tempfile

import numpy as np
import pytest
import torch

from predicitivecoding_b200.io import checkpoint as ck
from predicitivecoding_b200.llm.data import CorpusSource, StreamingTextDataset
from predicitivecoding_b200.llm.eval import fnv1a_tokens, held_out_hashed, training_split_hashed
from predicitivecoding_b200.llm.facade import PredictiveLlm
from predicitivecoding_b200.llm.generation import (ContinuousBatcher, Sampler, SamplingOptions, greedy,
                                                   self_speculative)
from predicitivecoding_b200.llm.options import GenerationOptions, TrainingOptions
from predicitivecoding_b200.llm.serving import export
from predicitivecoding_b200.llm.tokenizer import BpeTokenizer, ByteTokenizer, WordPieceTokenizer, split_pieces
from predicitivecoding_b200.models.config import DecoderLmConfig
from predicitivecoding_b200.models.decoder_lm import DecoderLM
from predicitivecoding_b200.optim.adam import LrSchedule

# directory of the reference project's Translate.Cli (its out-sample fixture); the test skips when unset
REF = os.environ.get("PCB_REFERENCE_TRANSLATE_CLI", "")
TEXT = ("the cat sat on the mat.\nthe dog sat on the log.\na bird sang in the tree.\n" * 6).strip()


def test_byte_tokenizer_roundtrip_and_specials():
    t = ByteTokenizer()
    ids = t.encode("héllo", add_bos=True, add_eos=True)
    assert ids[0] == 256 and ids[-1] == 257 and t.vocab_size == 260
    assert t.decode(ids) == "héllo"


def test_bpe_whole_stream_and_file_format():
    tok = BpeTokenizer()
    tok.train("abababab cdcdcd abab", 5)
    assert tok.vocab_size > 260
    s = "abab cd"
    assert tok.decode(tok.encode(s)) == s
    b = tok.save_to_bytes()
    assert int.from_bytes(b[:4], "little") == 0x42504531
    tok2 = BpeTokenizer.load_bytes(b)
    assert tok2.encode(s) == tok.encode(s)


def test_bpe_word_split_training_is_deterministic():
    lines = TEXT.split("\n")
    a, b = BpeTokenizer(), BpeTokenizer()
    a.train_from_corpus(lines, 300)
    b.train_from_corpus(lines, 300)
    assert a.merges_in_rank_order() == b.merges_in_rank_order()
    assert a.save_to_bytes()[:4] == (0x42504532).to_bytes(4, "little")
    assert a.decode(a.encode("the cat sat")) == "the cat sat"
    assert split_pieces("hi  there, you") == ["hi", " ", " there", ",", " you"]


def test_wordpiece():
    wp = WordPieceTokenizer.train(TEXT.split("\n"), 200)
    assert wp.decode(wp.encode("the cat sat")) == "the cat sat"


def test_streaming_windows_shift_by_one():
    ws = list(StreamingTextDataset(["abcdefgh"], ByteTokenizer(), 4, 2).windows())
    assert ws[0][0] == list(b"abcd") and ws[0][1] == list(b"bcde")
    assert ws[1][0] == list(b"cdef")


def test_fnv1a_split_is_content_hashed():
    w = ([1, 2, 3], [2, 3, 4])
    assert fnv1a_tokens([]) == 2166136261
    h = fnv1a_tokens([1])
    assert h == ((((((2166136261 ^ 1) * 16777619) & 0xFFFFFFFF) * 16777619 & 0xFFFFFFFF) * 16777619 & 0xFFFFFFFF)
                 * 16777619) & 0xFFFFFFFF
    ws = [([i, i + 1], [i + 1, i + 2]) for i in range(50)]
    ho, tr = list(held_out_hashed(ws, 5)), list(training_split_hashed(ws, 5))
    assert len(ho) + len(tr) == 50 and ho


def test_lr_schedule():
    s = LrSchedule(1.0, 0.1, 10, 100)
    assert s.at(0) == pytest.approx(0.1) and s.at(9) == pytest.approx(1.0)
    assert s.at(100) == 0.1 and 0.1 < s.at(50) < 1.0


def test_sampler_greedy_topk_and_penalties():
    logits = torch.tensor([1.0, 3.0, 2.0])
    assert Sampler(0).sample(logits, [], SamplingOptions(greedy=True)) == 1
    assert Sampler(0).sample(logits, [1], SamplingOptions(greedy=True, repetition_penalty=10.0)) == 2
    draws = {Sampler(s).sample(logits, [], SamplingOptions(top_k=1)) for s in range(10)}
    assert draws == {1}


def test_self_speculative_equals_greedy():
    cfg = DecoderLmConfig(64, 32, 2, 2, 64, 48, mtp_weight=0.3)
    m = DecoderLM(cfg, seed=3).eval()
    prompt = [1, 2, 3, 4]
    run = self_speculative(m, prompt, 20)
    assert run.tokens == greedy(m, prompt, 20)
    assert run.forwards <= 20


@pytest.mark.parametrize("cfg", [
    DecoderLmConfig(64, 32, 2, 2, 64, 48, use_rms_norm=True, use_rope=True, ffn="swiglu"),
    DecoderLmConfig(64, 32, 2, 2, 64, 48),
])
def test_kv_cache_serving_equals_full_forward(cfg):
    m = DecoderLM(cfg, seed=5).eval()
    inf = export(m, "cpu", torch.float32)
    prompts = [[1, 2, 3, 4, 5], [7, 8, 9, 10, 11]]
    out = inf.generate(prompts, 10)
    for p, o in zip(prompts, out):
        assert greedy(m, p, 10)[len(p):] == o


def test_continuous_batcher():
    cb = ContinuousBatcher(lambda seqs: [s[-1] + 1 for s in seqs], slots=2, eos=-1)
    ids = [cb.submit([i], 3) for i in range(5)]
    res = cb.run()
    assert res[ids[2]] == [3, 4, 5]


def test_facade_train_generate_eval_save_load():
    llm = PredictiveLlm.create_pc(dim=32, blocks=2, heads=2, ff_dim=64, max_seq=64)
    rep = llm.train(TEXT, TrainingOptions(epochs=3, batch_windows=4, peak_lr=0.01))
    assert rep.perplexity_after < rep.perplexity_before
    bpb = llm.evaluate_bits_per_byte(TEXT)
    assert 0 < bpb.bits_per_byte < 10 and bpb.bytes > 0
    text = llm.generate("the cat", 8)
    assert isinstance(text, str)
    llm.remember("the sky is blue")
    rep2 = llm.learn("the dog sat on the log.", steps=2)
    assert rep2.loss_after <= rep2.loss_before + 1e-4
    with tempfile.TemporaryDirectory() as d:
        llm.save(d)
        assert ck.is_checkpoint(d)
        back = PredictiveLlm.load(d)
        for a, b in zip(llm.model.parameters(), back.model.parameters()):
            assert torch.equal(a, b)
        assert back.memory.count == 1 and back.odometer.total == llm.odometer.total
        assert back.generate("the cat", 8) == llm.generate("the cat", 8)
    chat = llm.start_chat("be brief")
    assert isinstance(chat.say("hello"), str)
    with tempfile.TemporaryDirectory() as d:
        assert os.path.exists(llm.report(os.path.join(d, "r.html")))


def test_facade_bpe_tokenizer_travels_with_checkpoint():
    llm = PredictiveLlm.create_2026(dim=32, blocks=2, heads=2, ff_dim=32, max_seq=32, tokenizer_corpus=TEXT,
                                    merges=20)
    with tempfile.TemporaryDirectory() as d:
        llm.save(d, "bfloat16")
        back = PredictiveLlm.load(d)
        assert back.tokenizer.merges_in_rank_order() == llm.tokenizer.merges_in_rank_order()
        for a, b in zip(llm.model.parameters(), back.model.parameters()):
            assert torch.allclose(a, b, rtol=1e-2, atol=1e-3)


def test_learn_pc_ipc_runs():
    llm = PredictiveLlm.create_pc(dim=32, blocks=2, heads=2, ff_dim=64, max_seq=64)
    llm.pc_anchor_every = 2
    rep = llm.learn_pc("the cat sat on the mat. the dog sat on the log.", steps=2)
    assert math.isfinite(rep.loss_after) and llm.weights_are_finite()


@pytest.mark.parametrize("precision", ["float32", "half", "bfloat16", "int8"])
def test_tensor_blob_roundtrip(precision):
    t = torch.randn(5, 7)
    a, p = ck.read_tensor_blob(ck.tensor_blob(t, precision))
    assert p == precision and a.shape == (5, 7)
    tol = {"float32": 0, "half": 1e-3, "bfloat16": 1e-2, "int8": 2e-2}[precision]
    assert np.abs(a - t.numpy()).max() <= tol * np.abs(t.numpy()).max() + 1e-7


def test_opt1_and_dam1_roundtrip():
    ps = [torch.randn(3, 4), torch.randn(5)]
    mv = [(torch.randn(3, 4), torch.rand(3, 4)), None]
    with tempfile.TemporaryDirectory() as d:
        ck.save_opt1(os.path.join(d, "optimizer.bin"), ps, 7, mv)
        t, back = ck.load_opt1(os.path.join(d, "optimizer.bin"), ps)
        assert t == 7 and torch.equal(back[0][0], mv[0][0]) and float(back[1][0].abs().sum()) == 0
        ck.save_dam1(os.path.join(d, "adam-device.bin"), 3, [(np.ones(4), np.zeros(4))])
        t2, b2 = ck.load_dam1(os.path.join(d, "adam-device.bin"), [4])
        assert t2 == 3 and b2[0][0].sum() == 4


@pytest.mark.skipif(not REF or not os.path.exists(REF + "/out-sample/model.ckpt"),
                    reason="PCB_REFERENCE_TRANSLATE_CLI does not point at the reference fixture")
def test_golden_reference_translation_model():
    """The reference's own trained LLM1 model + BPE1 tokenizer, run through our DecoderLM,
    reproduces every translation pair it was trained on (LayerNorm, sinusoidal positions, GELU)."""
    cfg = DecoderLmConfig.from_json(open(REF + "/out-sample/manifest.json").read())
    m = DecoderLM(cfg)
    m.load_reference_parameters(ck.read_llm1(REF + "/out-sample/model.ckpt"))
    m.eval()
    tok = BpeTokenizer.load(REF + "/out-sample/tokenizer.bpe")
    ok = n = 0
    for line in open(REF + "/data/sample.tsv"):
        if line.startswith("#") or not line.strip():
            continue
        tag, src, tgt = line.rstrip("\n").split("\t")
        ids = [tok.bos] + tok.encode(f">>{tag}<< {src}\n")
        gen = greedy(m, ids, 12, eos=tok.eos)[len(ids):]
        if gen and gen[-1] == tok.eos:
            gen = gen[:-1]
        ok += tok.decode(gen) == tgt
        n += 1
    assert n > 0 and ok == n

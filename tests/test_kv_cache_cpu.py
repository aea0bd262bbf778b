"""GptModel KV caches, property by property (the checks of PredictiveCoding.UnitTests/LlmKvCacheTests.cs
and the recurrent-cache half of LlmHybridTests.cs, restated for this model)."""
import pytest
import torch

from predicitivecoding_b200.llm.gpt import GptModel, TransformerConfig


def cfg(**kw):
    base = dict(vocab_size=40, max_seq_len=64, embed_dim=32, num_heads=4, num_layers=2, feed_forward_dim=64,
                positional="rotary", norm="rmsnorm")
    base.update(kw)
    return TransformerConfig(**base)


SEQ = torch.tensor([3, 17, 5, 9, 22, 1, 30, 8, 14, 2, 27, 11])


def decode_logits(model, tokens):
    cache = model.create_cache()
    out = []
    with torch.no_grad():
        for p, t in enumerate(tokens.tolist()):
            out.append(model.step(t, p, cache))
    return torch.stack(out), cache


def test_window_larger_than_the_sequence_is_identical_to_full_attention():
    full = GptModel(cfg(), seed=1)
    windowed = GptModel(cfg(window_size=64), seed=1)
    a, _ = decode_logits(full, SEQ)
    b, _ = decode_logits(windowed, SEQ)
    assert torch.equal(a, b)


def test_eviction_keeps_the_sinks_and_the_newest_window():
    m = GptModel(cfg(window_size=4, num_sink_tokens=2), seed=2)
    _, cache = decode_logits(m, SEQ)
    for layer in cache.layers:
        assert layer.positions == [0, 1] + list(range(len(SEQ) - 4, len(SEQ)))
        assert layer.k.shape[2] == 6


def test_cache_bytes_plateau_once_the_window_is_full():
    m = GptModel(cfg(window_size=4, num_sink_tokens=1), seed=3)
    cache = m.create_cache()
    sizes = []
    with torch.no_grad():
        for p, t in enumerate(SEQ.tolist()):
            m.step(t, p, cache)
            sizes.append(cache.bytes_used)
    assert sizes[0] < sizes[4]
    assert len(set(sizes[5:])) == 1            # sinks + window entries from then on


def test_half_cache_halves_the_bytes_and_stays_close():
    a, ca = decode_logits(GptModel(cfg(), seed=4), SEQ)
    b, cb = decode_logits(GptModel(cfg(kv_cache_half=True), seed=4), SEQ)
    assert cb.bytes_used * 2 == ca.bytes_used
    assert float((a - b).abs().max()) < 1e-2 * float(a.abs().max())


def test_latent_cache_reports_its_bytes():
    m = GptModel(cfg(attention="latent", kv_latent_dim=16, rope_head_dim=8), seed=5)
    _, cache = decode_logits(m, SEQ[:6])
    assert cache.bytes_used > 0
    dense = GptModel(cfg(), seed=5)
    _, dcache = decode_logits(dense, SEQ[:6])
    assert cache.bytes_used < dcache.bytes_used            # the point of the compressed latent


def test_invalid_window_configs_raise():
    with pytest.raises(ValueError):
        cfg(window_size=-1).validate()
    with pytest.raises(ValueError):
        cfg(num_sink_tokens=2).validate()                    # sinks need a window
    with pytest.raises(ValueError):
        cfg(window_size=8, attention="latent").validate()


def test_recurrent_layer_state_stays_constant_while_attention_grows():
    m = GptModel(cfg(positional="sinusoidal", norm="layernorm", block_pattern="AT"), seed=6)
    cache = m.create_cache()
    attn, rec = [], []
    with torch.no_grad():
        for p, t in enumerate(SEQ.tolist()):
            m.step(t, p, cache)
            attn.append(cache.layers[0].bytes_used)
            rec.append(cache.layers[1].bytes_used)
    assert attn[-1] > attn[0]
    assert len(set(rec)) == 1


def test_cached_decoding_equals_the_full_forward():
    m = GptModel(cfg(num_kv_heads=2), seed=7)
    steps, _ = decode_logits(m, SEQ)
    with torch.no_grad():
        full = m(SEQ[None])[0]
    assert torch.allclose(steps, full, atol=1e-5, rtol=1e-4)

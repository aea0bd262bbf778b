"""Tensor-parallel KV-cache decoding: greedy tokens agree with the fp32 reference model (1 and 2 GPUs)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _cfg():
    from predicitivecoding_b200.models.config import DecoderLmConfig
    return DecoderLmConfig(vocab=512, dim=256, num_blocks=2, num_heads=4, ff_dim=512, max_seq=512,
                           use_rms_norm=True, use_rope=True, ffn="swiglu")


def _prompt():
    g = torch.Generator().manual_seed(77)
    return torch.randint(0, 512, (2, 128), generator=g)


def _check_greedy(tokens, model, prompt):
    """Every generated token must be (within bf16 noise) the argmax of the fp32 model on its own prefix."""
    seq = torch.cat((prompt, tokens), 1).cuda()
    with torch.no_grad():
        logits = model.cuda()(seq[:, :-1]).float()[:, prompt.shape[1] - 1:]     # predictions for the new tokens
    chosen = logits.gather(-1, seq[:, prompt.shape[1]:, None].cuda()).squeeze(-1)
    best = logits.max(-1).values
    spread = logits.std(-1)
    assert bool(((best - chosen) <= 0.05 * spread).all()), (best - chosen) / spread


def _run(rank, world, q=None, port=None):
    import torch.distributed as dist
    from datetime import timedelta
    pg = None
    if world > 1:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                timeout=timedelta(seconds=60))
        pg = dist.group.WORLD
    dec = None
    try:
        from predicitivecoding_b200.llm.tp_decode import TensorParallelDecoder
        from predicitivecoding_b200.models.decoder_lm import DecoderLM
        cfg = _cfg()
        model = DecoderLM(cfg, seed=3)
        dec = TensorParallelDecoder(cfg, batch=2, capacity=256, process_group=pg,
                                    device=torch.device("cuda", rank), model=model, use_graph=True)
        toks = dec.generate(_prompt(), 12)
        dec.check()
        if q is not None:
            q.put((rank, toks))
        return toks, model
    finally:
        if dec is not None:
            dec.release()
        if world > 1:
            dist.destroy_process_group()


def test_tp_decode_single_gpu_matches_reference():
    toks, model = _run(0, 1)
    assert toks.shape == (2, 12)
    _check_greedy(toks, model, _prompt())


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_decode_matches_reference():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_run, args=(r, world, q, port)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert torch.equal(res[0], res[1])            # every rank samples the same tokens
    from predicitivecoding_b200.models.decoder_lm import DecoderLM
    _check_greedy(res[0], DecoderLM(_cfg(), seed=3), _prompt())

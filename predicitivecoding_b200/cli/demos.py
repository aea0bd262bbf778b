"""Demo menu: the reference's 13 demos mapped onto this framework, runnable headless.

Reference: PredictiveCoding.Main/Program.cs and Demos/*.cs (synthetic classification, the
Millidge-style PC classifier, CIFAR, temporal sequences, mixture of experts, faces, language ID,
people counting, Thousand Brains, the full LLM, LM distillation, web corpus, web pretraining on
the GPU).  Demos that need external data or network access run on synthetic stand-ins.
"""
from __future__ import annotations

import sys
from typing import Optional

import torch


def synthetic() -> str:
    from ..pc.network import Network, NetworkConfig
    from ..pc.trainer import SyntheticDataset, Trainer, TrainingConfig
    tr, te = SyntheticDataset.split(num_classes=4, input_dim=20, total_per_class=100)
    cfg = NetworkConfig(layer_sizes=(20, 32, 4), weight_lr=0.01)
    net = Network(cfg, seed=0)
    Trainer(net, TrainingConfig(network=cfg, epochs=5, inference_steps=10)).train(tr, te)
    acc = sum(net.predict(x, 10) == int(y.argmax()) for x, y in zip(te.inputs, te.labels)) / len(te.labels)
    return f"synthetic PC classifier: test accuracy {acc:.2f}"


def temporal() -> str:
    from ..pc.network import Network, NetworkConfig
    from ..pc.networks import TemporalNetwork
    tn = TemporalNetwork(Network(NetworkConfig(layer_sizes=(4, 8, 4)), seed=0), 0.5)
    seq = [torch.eye(4)[i] for i in (0, 1, 2, 3)] * 10
    for a, b in zip(seq, seq[1:]):
        tn.step(a, b, 10)
    return f"temporal: predicted class after a 0 -> {tn.predict(seq[0], 10)}"


def moe() -> str:
    from ..pc.network import NetworkConfig
    from ..pc.networks import MixtureOfExperts, MixtureOfExpertsConfig
    m = MixtureOfExperts(MixtureOfExpertsConfig(
        expert_count=3, expert_config=NetworkConfig(layer_sizes=(6, 8, 3), weight_lr=0.05)))
    for i in range(90):
        m.learn(torch.eye(6)[i % 3], torch.eye(3)[i % 3], 10)
    return f"mixture of experts: classes of e0..e2 -> {[m.predict(torch.eye(6)[k], 10) for k in range(3)]}"


def language_id() -> str:
    from ..systems.data import NGramLanguageClassifierTrainer
    t = NGramLanguageClassifierTrainer()
    t.add("en", "the house is big and the garden is green")
    t.add("it", "la casa e grande e il giardino e verde")
    return f"language id: 'the garden' -> {t.train().predict('the garden')}"


def people_counting() -> str:
    from ..systems import vision as vi
    from ..systems.imaging import RgbImage
    frames = [RgbImage(64, 64) for _ in range(6)]
    pipe = vi.PeopleCountingPipeline(lambda f: [vi.Detection(10, 10, 20, 40)], vi.SortTracker(min_hits=2))
    r = [pipe.process(f) for f in frames][-1]
    return f"people counting: current {r.current_count}, unique {r.unique_count}"


def thousand_brains() -> str:
    from ..systems import brain as br
    data = br.SyntheticObjectDataset(n_objects=5, points=8)
    rep = br.recognition_benchmark(br.ThousandBrainsSystem(data.size, data.size), data, noise=0.05)
    return f"thousand brains: recognition accuracy {rep.accuracy:.2f}"


def llm() -> str:
    from ..llm.facade import PredictiveLlm
    from ..llm.options import TrainingOptions
    text = "the cat sat on the mat.\nthe dog sat on the log.\n" * 10
    lm = PredictiveLlm.create_pc(dim=32, blocks=1, heads=2, ff_dim=64, max_seq=64)
    rep = lm.train(text, TrainingOptions(epochs=2, batch_windows=4))
    return f"LLM: perplexity {rep.perplexity_before:.1f} -> {rep.perplexity_after:.1f}; sample: {lm.generate('the', 8)!r}"


def millidge() -> str:
    """MillidgeReview2022Demo: free-energy convergence during inference, accuracy vs inference steps,
    depth comparison and noise robustness on a synthetic 4-class task."""
    from ..pc.network import Network, NetworkConfig
    from ..pc.trainer import SyntheticDataset, Trainer, TrainingConfig

    def data(noise):
        return SyntheticDataset.split(num_classes=4, input_dim=20, total_per_class=60, noise=noise, seed=42)

    def train(sizes, tr, epochs=6):
        cfg = NetworkConfig(layer_sizes=sizes, weight_lr=0.01)
        net = Network(cfg, seed=42)
        Trainer(net, TrainingConfig(network=cfg, epochs=epochs, inference_steps=20)).train(tr, None)
        return net

    def acc(net, te, steps=20):
        return sum(net.predict(x, steps) == int(y.argmax()) for x, y in zip(te.inputs, te.labels)) / len(te.labels)

    tr, te = data(0.35)
    ref = train((20, 64, 32, 4), tr)
    trace = torch.tensor([ref.infer_trace(x, 30) for x in te.inputs[:20]]).mean(0)
    lines = [f"energy T=1 {float(trace[0]):.3f} -> T=30 {float(trace[-1]):.3f}"]
    lines.append("accuracy by inference steps: " + ", ".join(f"T={t}:{acc(ref, te, t):.2f}" for t in (1, 5, 20)))
    lines.append("depth: " + ", ".join(f"{len(s) - 2} hidden:{acc(train(s, tr, 4), te):.2f}"
                                       for s in ((20, 4), (20, 32, 4), (20, 64, 32, 4))))
    lines.append("noise: " + ", ".join(f"{n}:{acc(train((20, 32, 4), data(n)[0], 4), data(n)[1]):.2f}"
                                       for n in (0.1, 0.5)))
    return "Millidge review experiments: " + "; ".join(lines)


def hard_classification() -> str:
    """HardClassificationDemo (CIFAR stand-in): a deeper PC classifier on 10 overlapping classes of
    3x8x8 inputs; CIFAR-10 batches load through systems.data.load_cifar10 when present."""
    from ..pc.network import Network, NetworkConfig
    from ..pc.trainer import SyntheticDataset, Trainer, TrainingConfig
    tr, te = SyntheticDataset.split(num_classes=10, input_dim=192, total_per_class=30, noise=0.6, seed=3)
    cfg = NetworkConfig(layer_sizes=(192, 128, 64, 10), weight_lr=0.005)
    net = Network(cfg, seed=1)
    Trainer(net, TrainingConfig(network=cfg, epochs=4, inference_steps=15)).train(tr, None)
    a = sum(net.predict(x, 15) == int(y.argmax()) for x, y in zip(te.inputs, te.labels)) / len(te.labels)
    return f"hard classification (10 classes, 192-D): test accuracy {a:.2f} (chance 0.10)"


def faces() -> str:
    """FaceRecognitionDemo on synthetic identities: LBP and PC-latent embedders, verification accuracy."""
    import numpy as np
    from ..systems.faces import LbpEmbedder, verification_benchmark
    from ..systems.imaging import RgbImage
    rng = np.random.default_rng(0)
    base = [rng.integers(0, 255, (64, 64, 3)) for _ in range(6)]
    shot = lambda i: RgbImage.from_pixel_data(np.clip(base[i] + rng.normal(0, 25, base[i].shape), 0, 255)
                                              .astype(np.uint8), 64, 64)
    pairs = [(shot(i), shot(i), True) for i in range(6)] + [(shot(i), shot((i + 1) % 6), False) for i in range(6)]
    r = verification_benchmark(LbpEmbedder(), pairs, folds=2)
    return f"faces (LBP, synthetic identities): verification accuracy {r.accuracy:.2f}, AUC {r.auc_roc:.2f}"


def lm_distillation() -> str:
    """LmDistillationDemo: a small LLM learns a teacher's answers (the teacher is a rule here)."""
    from ..llm.facade import PredictiveLlm
    lm = PredictiveLlm.create_pc(dim=32, blocks=1, heads=2, ff_dim=64, max_seq=64)
    teacher = lambda prompt: prompt[::-1][:8]
    loss = lm.distill_from(teacher, ["abc", "hello", "stop"], steps=6)
    return f"LM distillation: final distillation loss {loss:.3f}"


def web_corpus(directory: str = "", pages: Optional[dict] = None) -> str:
    """WebCorpusDemo: crawl (here a recorded site) and sediment the kept pages into corpus shards."""
    import tempfile
    from ..systems.data import ShardedCorpusWriter
    from ..systems.data_sources import CrawlOptions, WebCrawler
    para = "<p>" + " ".join(f"w{i}" for i in range(80)) + "</p>"
    site = pages or {"http://site.test/": ("text/html", f"<title>t</title>{para}<a href='/b'>b</a>"),
                     "http://site.test/b": ("text/html", para.replace("w", "v"))}
    out = directory or tempfile.mkdtemp(prefix="web-corpus-")
    writer = ShardedCorpusWriter(out)
    rep = WebCrawler(lambda u: site[u], CrawlOptions(per_host_delay=0)).crawl(
        list(site)[:1], lambda p: writer.append(p.blocks))
    writer.close()
    return f"web corpus: {rep.pages_kept} pages kept of {rep.pages_fetched} fetched -> {out}"


def web_pretrain(root: str = "", max_steps: int = 20) -> str:
    """WebPretrainDemo (the device path end to end): corpus shards -> BPE -> Small preset -> the fused
    device trainer through engine.pretrainer, with checkpoints; a second run resumes from the model
    directory, recognised by the checkpoint's own format marker."""
    import os
    import tempfile
    from ..engine.pretrainer import DevicePretrainOptions, pretrain
    from ..io.checkpoint import is_checkpoint
    from ..llm.data import CorpusSource
    from ..llm.facade import PredictiveLlm
    from ..llm.tokenizer import BpeTokenizer
    if not torch.cuda.is_available():
        return "web pretraining: no CUDA device visible (the run needs a GPU)"
    root = root or tempfile.mkdtemp(prefix="web-pretrain-")
    shards, model_dir = os.path.join(root, "web-corpus"), os.path.join(root, "web-model")
    if not os.path.isdir(shards) or not any(f.startswith("shard-") for f in os.listdir(shards)):
        web_corpus(shards)
    corpus = CorpusSource.from_folder(shards, "shard-*.txt").with_boilerplate_stripped().deduplicated()
    if is_checkpoint(model_dir):
        llm = PredictiveLlm.load(model_dir)
        how = "resumed"
    else:
        tok = BpeTokenizer()
        tok.train_from_corpus(corpus.lines(), target_vocab=512)
        llm = PredictiveLlm.create_small(tok, max_seq=128)
        how = "fresh"
    rep = pretrain(llm, corpus, DevicePretrainOptions(epochs=100, seq_len=128, stride=128, micro_batch_windows=4,
                                                      max_steps=max_steps, eval_every_steps=10, eval_windows=4,
                                                      checkpoint_dir=model_dir, checkpoint_every_steps=10,
                                                      log_path=os.path.join(model_dir, "train.jsonl")))
    return (f"web pretraining ({how}): {rep.steps} steps, {rep.tokens} tokens, final eval loss "
            f"{rep.final_eval_loss:.3f}; checkpoint {model_dir}")


DEMOS = {"1": ("synthetic PC classification", synthetic), "2": ("Millidge review experiments", millidge),
         "3": ("hard classification (CIFAR stand-in)", hard_classification), "4": ("temporal sequences", temporal),
         "5": ("mixture of experts", moe), "6": ("face recognition", faces),
         "7": ("language identification", language_id), "8": ("people counting", people_counting),
         "9": ("thousand brains", thousand_brains), "10": ("predictive LLM", llm),
         "11": ("LM distillation", lm_distillation), "12": ("web corpus", web_corpus),
         "13": ("web pretraining on the GPU", web_pretrain)}


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if not argv:
        for k, (name, _) in DEMOS.items():
            print(f"{k:>3}  {name}")
        print("run: python -m predicitivecoding_b200.cli.demos <number>")
        return 0
    for k in argv:
        print(DEMOS[k][1]())
    return 0


if __name__ == "__main__":
    sys.exit(main())

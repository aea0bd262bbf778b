"""Demo menu: the reference's 13 demos mapped onto this framework, runnable headless.

Reference: PredictiveCoding.Main/Program.cs and Demos/*.cs (synthetic classification, the
Millidge-style PC classifier, CIFAR, temporal sequences, mixture of experts, faces, language ID,
people counting, Thousand Brains, the full LLM, LM distillation, web corpus, web pretraining on
the GPU).  Demos that need external data or network access run on synthetic stand-ins.
"""
from __future__ import annotations

import sys

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


DEMOS = {"1": ("synthetic PC classification", synthetic), "4": ("temporal sequences", temporal),
         "5": ("mixture of experts", moe), "7": ("language identification", language_id),
         "8": ("people counting", people_counting), "9": ("thousand brains", thousand_brains),
         "10": ("predictive LLM", llm)}


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

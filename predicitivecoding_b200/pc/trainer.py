"""PC training loop, datasets and metric logging.

Reference: PredicitiveCoding/Training/Trainer.cs:35-176, TrainingConfig.cs:13-69,
Batch.cs:18, Data/IDataset.cs:13, Data/SyntheticDataset.cs:21-164,
Logging/MetricLogger.cs:11-122, Logging/CsvLogger.cs:10-56.

``Trainer.train_epoch`` calls ``Network.learn`` per sample (the reference's online
rule); ``Trainer.train_epoch_batched`` runs the same epoch through the batched
engine (batch-mean Hebbian update, CPU oracle or fused GPU engine).
"""
from __future__ import annotations

import csv
import os
import time
from dataclasses import dataclass, field
from typing import Iterator, List, Optional, Sequence

import torch

from .network import Network, NetworkConfig


@dataclass
class TrainingConfig:
    network: NetworkConfig = field(default_factory=NetworkConfig)
    inference_steps: int = 20
    epochs: int = 50
    batch_size: int = 32
    seed: int = 42
    csv_output_path: Optional[str] = None
    log_every_n_epochs: int = 1

    def validate(self) -> None:
        self.network.validate()
        if self.inference_steps <= 0:
            raise ValueError("InferenceSteps must be > 0.")
        if self.epochs <= 0:
            raise ValueError("Epochs must be > 0.")
        if self.batch_size <= 0:
            raise ValueError("BatchSize must be > 0.")


@dataclass
class Batch:
    inputs: torch.Tensor   # [B, in]
    labels: torch.Tensor   # [B, classes] one-hot

    @property
    def size(self) -> int:
        return self.inputs.shape[0]


class SyntheticDataset:
    """Gaussian-blob classification data (Data/SyntheticDataset.cs:21-164)."""

    def __init__(self, inputs: torch.Tensor, labels: torch.Tensor, name: str):
        self.inputs, self.labels, self.name = inputs, labels, name

    @property
    def input_size(self) -> int:
        return self.inputs.shape[1]

    @property
    def label_count(self) -> int:
        return self.labels.shape[1]

    @property
    def total_samples(self) -> int:
        return self.inputs.shape[0]

    def get_batches(self, batch_size: int, gen: Optional[torch.Generator] = None) -> Iterator[Batch]:
        order = torch.randperm(self.total_samples, generator=gen) if gen is not None else torch.arange(self.total_samples)
        for i in range(0, self.total_samples, batch_size):
            idx = order[i:i + batch_size]
            yield Batch(self.inputs[idx], self.labels[idx])

    @staticmethod
    def split(num_classes: int = 4, input_dim: int = 20, total_per_class: int = 200, test_fraction: float = 0.2,
              noise: float = 0.4, seed: int = 42):
        gen = torch.Generator().manual_seed(seed)
        centers = torch.randn(num_classes, input_dim, generator=gen) * 2.0
        test_per = max(1, int(total_per_class * test_fraction))
        train_per = total_per_class - test_per
        xs_tr, ys_tr, xs_te, ys_te = [], [], [], []
        for c in range(num_classes):
            onehot = torch.zeros(num_classes)
            onehot[c] = 1.0
            x = centers[c] + noise * torch.randn(total_per_class, input_dim, generator=gen)
            xs_tr.append(x[:train_per]); ys_tr.append(onehot.expand(train_per, -1))
            xs_te.append(x[train_per:]); ys_te.append(onehot.expand(test_per, -1))
        train = SyntheticDataset(torch.cat(xs_tr), torch.cat(ys_tr).clone(),
                                 f"Train ({num_classes}cl x {train_per}={num_classes * train_per})")
        test = SyntheticDataset(torch.cat(xs_te), torch.cat(ys_te).clone(),
                                f"Test ({num_classes}cl x {test_per}={num_classes * test_per})")
        return train, test


@dataclass
class EpochMetrics:
    epoch: int
    train_energy: float
    train_accuracy: float
    test_energy: float
    test_accuracy: float
    weight_norm: float
    elapsed_seconds: float


class MetricLogger:
    """Console table of epoch metrics (Logging/MetricLogger.cs:11-122)."""

    def __init__(self, verbose: bool = True):
        self.history: List[EpochMetrics] = []
        self.verbose = verbose

    def log(self, m: EpochMetrics) -> None:
        self.history.append(m)
        if self.verbose:
            print(f"epoch {m.epoch:4d} | train F {m.train_energy:9.4f} acc {m.train_accuracy:6.2%} | "
                  f"test F {m.test_energy:9.4f} acc {m.test_accuracy:6.2%} | |W| {m.weight_norm:8.4f} | "
                  f"{m.elapsed_seconds:7.2f}s")


class CsvLogger:
    """Appends EpochMetrics rows to a CSV file (Logging/CsvLogger.cs:10-56)."""

    HEADER = ["Epoch", "TrainEnergy", "TrainAccuracy", "TestEnergy", "TestAccuracy", "WeightNorm", "ElapsedSeconds"]

    def __init__(self, path: str):
        self.path = path
        if not os.path.exists(path) or os.path.getsize(path) == 0:
            with open(path, "w", newline="") as f:
                csv.writer(f).writerow(self.HEADER)

    def log(self, m: EpochMetrics) -> None:
        with open(self.path, "a", newline="") as f:
            csv.writer(f).writerow([m.epoch, f"{m.train_energy:.6f}", f"{m.train_accuracy:.6f}", f"{m.test_energy:.6f}",
                                    f"{m.test_accuracy:.6f}", f"{m.weight_norm:.6f}", f"{m.elapsed_seconds:.3f}"])


class Trainer:
    """Epoch loop over a dataset (Training/Trainer.cs:35-176)."""

    def __init__(self, network: Network, config: TrainingConfig):
        config.validate()
        self.net, self.cfg = network, config
        self.gen = torch.Generator().manual_seed(config.seed)

    def train_epoch(self, data: SyntheticDataset) -> float:
        """Per-sample Learn over every batch; returns the mean energy after learning."""
        total, n = 0.0, 0
        for batch in data.get_batches(self.cfg.batch_size, self.gen):
            for i in range(batch.size):
                total += self.net.learn(batch.inputs[i], batch.labels[i], self.cfg.inference_steps)
                n += 1
        return total / max(n, 1)

    def train_epoch_batched(self, data: SyntheticDataset, engine) -> float:
        """One epoch through a batched engine (``BatchedPCReference`` or ``BatchedPC``)."""
        total, n = 0.0, 0
        for batch in data.get_batches(self.cfg.batch_size, self.gen):
            if hasattr(engine, "B") and batch.size != engine.B:
                continue
            out = engine.learn(batch.inputs, batch.labels, self.cfg.inference_steps)
            total += float(out) if out is not None else engine.energy_value()
            n += 1
        return total / max(n, 1)

    def evaluate(self, data: SyntheticDataset) -> tuple:
        """Energy-argmin prediction accuracy and mean winning energy (Trainer.cs:97-127)."""
        correct, energy = 0, 0.0
        for i in range(data.total_samples):
            c, e = self.net.predict_with_energy(data.inputs[i], self.cfg.inference_steps)
            correct += int(c == int(data.labels[i].argmax()))
            energy += e
        n = max(data.total_samples, 1)
        return energy / n, correct / n

    def train(self, train: SyntheticDataset, test: Optional[SyntheticDataset] = None,
              logger: Optional[MetricLogger] = None) -> List[EpochMetrics]:
        logger = logger or MetricLogger(verbose=False)
        csvlog = CsvLogger(self.cfg.csv_output_path) if self.cfg.csv_output_path else None
        t0 = time.time()
        for ep in range(1, self.cfg.epochs + 1):
            tr_e = self.train_epoch(train)
            if ep % self.cfg.log_every_n_epochs == 0 or ep == self.cfg.epochs:
                _, tr_acc = self.evaluate(train)
                te_e, te_acc = self.evaluate(test) if test is not None else (0.0, 0.0)
                m = EpochMetrics(ep, tr_e, tr_acc, te_e, te_acc, self.net.average_weight_norm(), time.time() - t0)
                logger.log(m)
                if csvlog:
                    csvlog.log(m)
        return logger.history

"""Synthetic, index-addressable datasets and the topology-aware batch sampler.

Every sample is a pure function of ``(seed, index)``, so any rank can produce
any sample and a resumed run replays the same data (reference
``src/hybrid_training/training/data.py:63-503``).  The sampler draws one
permutation per epoch and gives each ``dp_shard`` rank its slice of every
global batch; tensor/sequence-parallel peers (same ``dp_shard`` coordinate)
receive identical batches.

Token datasets produce either the reference's noisy affine recurrence or
uniform random tokens (the benchmark distribution).  Batches destined for a
GPU are assembled in pinned host memory so the host-to-device copy is
asynchronous.
"""

from __future__ import annotations

from collections.abc import Iterator
from dataclasses import dataclass

import torch

from ..config import DataConfig, ModelConfig
from ..distributed.groups import GroupHandle
from ..errors import ConfigurationError, format_error
from ..utils.reproducibility import derive_seed

__all__ = ["Batch", "DistributedBatchSampler", "SyntheticDataLoader", "SyntheticDataset", "SyntheticMLPDataset",
           "SyntheticTokenDataset", "build_dataset"]


@dataclass
class Batch:
    inputs: torch.Tensor
    targets: torch.Tensor
    indices: tuple[int, ...]

    def to(self, device: torch.device) -> Batch:
        return Batch(self.inputs.to(device, non_blocking=True), self.targets.to(device, non_blocking=True), self.indices)

    @property
    def size(self) -> int:
        return int(self.inputs.shape[0])


class SyntheticDataset:
    def __init__(self, num_samples: int, seed: int) -> None:
        if num_samples < 1:
            raise ConfigurationError(format_error("data.SyntheticDataset", "a synthetic dataset has one or more samples", expected=">= 1",
                                                  observed=num_samples, resolution="increase the sample count in the data config"))
        self._num_samples, self._seed = num_samples, seed
        self.pin_memory = False

    def __len__(self) -> int:
        return self._num_samples

    def _generator(self, index: int) -> torch.Generator:
        g = torch.Generator()
        g.manual_seed(derive_seed(self._seed, "sample", index))
        return g

    def get(self, index: int) -> tuple[torch.Tensor, torch.Tensor]:
        raise NotImplementedError

    def batch(self, indices: tuple[int, ...]) -> Batch:
        samples = [self.get(i) for i in indices]
        x = torch.stack([s[0] for s in samples])
        y = torch.stack([s[1] for s in samples])
        if self.pin_memory:
            x, y = x.pin_memory(), y.pin_memory()
        return Batch(x, y, tuple(indices))


class SyntheticMLPDataset(SyntheticDataset):
    """Regression targets from a fixed random teacher MLP plus noise."""

    def __init__(self, num_samples: int, seed: int, *, input_size: int, output_size: int, hidden_size: int = 32,
                 noise_std: float = 0.01) -> None:
        super().__init__(num_samples, seed)
        self.input_size, self.output_size, self.noise_std = input_size, output_size, noise_std
        teacher = torch.Generator()
        teacher.manual_seed(derive_seed(seed, "teacher"))
        self._a = torch.randn(input_size, hidden_size, generator=teacher) / input_size**0.5
        self._b = torch.randn(hidden_size, output_size, generator=teacher) / hidden_size**0.5

    def get(self, index: int) -> tuple[torch.Tensor, torch.Tensor]:
        g = self._generator(index)
        x = torch.randn(self.input_size, generator=g)
        y = torch.tanh(x @ self._a) @ self._b + self.noise_std * torch.randn(self.output_size, generator=g)
        return x, y


class SyntheticTokenDataset(SyntheticDataset):
    """Next-token pairs ``(tokens[:-1], tokens[1:])``.

    ``recurrence``: ``t[i] = (7 t[i-1] + 3) mod V`` with probability 0.9, a
    uniform token otherwise (learnable).  ``uniform``: i.i.d. uniform tokens.
    """

    def __init__(self, num_samples: int, seed: int, *, vocab_size: int, sequence_length: int, noise_probability: float = 0.1,
                 distribution: str = "recurrence") -> None:
        super().__init__(num_samples, seed)
        if sequence_length < 2:
            raise ConfigurationError(format_error("data.SyntheticTokenDataset", "next-token prediction needs two positions",
                                                  expected=">= 2", observed=sequence_length, resolution="raise sequence_length"))
        self.vocab_size, self.sequence_length = vocab_size, sequence_length
        self.noise_probability, self.distribution = noise_probability, distribution

    def get(self, index: int) -> tuple[torch.Tensor, torch.Tensor]:
        g = self._generator(index)
        n = self.sequence_length + 1
        if self.distribution == "uniform":
            tokens = torch.randint(0, self.vocab_size, (n,), generator=g)
        else:
            first = int(torch.randint(0, self.vocab_size, (1,), generator=g))
            noise = torch.rand(n, generator=g).tolist()
            rand = torch.randint(0, self.vocab_size, (n,), generator=g).tolist()
            seq = [first]
            v, p = self.vocab_size, self.noise_probability
            for i in range(1, n):
                seq.append(rand[i] if noise[i] < p else (7 * seq[-1] + 3) % v)
            tokens = torch.tensor(seq, dtype=torch.long)
        return tokens[:-1].contiguous(), tokens[1:].contiguous()


def build_dataset(model_config: ModelConfig, data_config: DataConfig, *, split: str = "train") -> SyntheticDataset:
    if split not in ("train", "eval"):
        raise ConfigurationError(format_error("data.build_dataset", "unknown split", expected=["train", "eval"], observed=split,
                                              resolution="the splits are 'train' and 'eval'"))
    n = data_config.num_train_samples if split == "train" else data_config.num_eval_samples
    seed = derive_seed(data_config.seed, f"dataset-{split}")
    if model_config.kind == "transformer":
        return SyntheticTokenDataset(max(n, 1), seed, vocab_size=model_config.vocab_size, sequence_length=data_config.sequence_length,
                                     distribution=data_config.token_distribution)
    return SyntheticMLPDataset(max(n, 1), seed, input_size=model_config.input_size, output_size=model_config.output_size)


class DistributedBatchSampler:
    """Per-epoch permutation; ``dp_shard`` rank ``r`` takes micro-batch slice ``r`` of each global batch."""

    def __init__(self, dataset_size: int, micro_batch_size: int, data_group: GroupHandle, *, shuffle: bool = True, seed: int = 0,
                 drop_last: bool = True) -> None:
        self.dataset_size, self.micro_batch_size, self.data_group = dataset_size, micro_batch_size, data_group
        self.shuffle, self.seed, self.drop_last = shuffle, seed, drop_last
        self.global_batch_size = micro_batch_size * data_group.size
        if dataset_size < self.global_batch_size:
            raise ConfigurationError(format_error("data.DistributedBatchSampler", "there are fewer samples than one step consumes",
                                                  rank=data_group.global_rank, expected=f">= {self.global_batch_size} samples",
                                                  observed=dataset_size, resolution="raise num_train_samples or lower micro_batch_size"))

    @property
    def batches_per_epoch(self) -> int:
        return self.dataset_size // self.global_batch_size

    def epoch_order(self, epoch: int) -> torch.Tensor:
        if not self.shuffle:
            return torch.arange(self.dataset_size)
        g = torch.Generator()
        g.manual_seed(derive_seed(self.seed, "shuffle", epoch))
        return torch.randperm(self.dataset_size, generator=g)

    def __iter__(self) -> Iterator[tuple[int, ...]]:
        return self.iter_epoch(0)

    def iter_epoch(self, epoch: int) -> Iterator[tuple[int, ...]]:
        order = self.epoch_order(epoch).tolist()
        lo = self.data_group.local_rank * self.micro_batch_size
        for b in range(self.batches_per_epoch):
            start = b * self.global_batch_size + lo
            yield tuple(order[start:start + self.micro_batch_size])

    def global_batch_indices(self, epoch: int, batch_index: int) -> tuple[int, ...]:
        order = self.epoch_order(epoch).tolist()
        start = batch_index * self.global_batch_size
        return tuple(order[start:start + self.global_batch_size])


class SyntheticDataLoader:
    def __init__(self, dataset: SyntheticDataset, sampler: DistributedBatchSampler, device: torch.device) -> None:
        self.dataset, self.sampler, self.device = dataset, sampler, device
        dataset.pin_memory = device.type == "cuda"

    def __len__(self) -> int:
        return self.sampler.batches_per_epoch

    def iter_epoch(self, epoch: int) -> Iterator[Batch]:
        for indices in self.sampler.iter_epoch(epoch):
            yield self.dataset.batch(indices).to(self.device)

    def iter_host(self, epoch: int) -> Iterator[Batch]:
        """Batches left in (pinned) host memory, for callers that stage the copy themselves."""
        for indices in self.sampler.iter_epoch(epoch):
            yield self.dataset.batch(indices)

    def global_batch(self, epoch: int, batch_index: int) -> Batch:
        return self.dataset.batch(self.sampler.global_batch_indices(epoch, batch_index)).to(self.device)

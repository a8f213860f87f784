"""Configuration types mirroring crates/klearu-core/src/config.rs:3-143."""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from enum import IntEnum

from . import _lib


class HashFunctionType(IntEnum):  # config.rs:3-10
    SimHash = _lib.HASH_SIMHASH
    WtaHash = _lib.HASH_WTA
    DwtaHash = _lib.HASH_DWTA
    MinHash = _lib.HASH_MINHASH
    SparseRandomProjection = _lib.HASH_SRP


class BucketType(IntEnum):  # config.rs:12-16
    Fifo = _lib.BUCKET_FIFO
    Reservoir = _lib.BUCKET_RESERVOIR


class SamplingType(IntEnum):  # config.rs:18-23
    Vanilla = _lib.SAMPLING_VANILLA
    TopK = _lib.SAMPLING_TOPK
    Threshold = _lib.SAMPLING_THRESHOLD


class ActivationType(IntEnum):  # config.rs:25-32
    Relu = _lib.ACT_RELU
    Sigmoid = _lib.ACT_SIGMOID
    Tanh = _lib.ACT_TANH
    Softmax = _lib.ACT_SOFTMAX
    Identity = _lib.ACT_IDENTITY


class OptimizerType(IntEnum):  # config.rs:34-38
    Sgd = _lib.OPT_SGD
    Adam = _lib.OPT_ADAM


@dataclass
class LshConfig:  # config.rs:40-65 (defaults included)
    hash_function: HashFunctionType = HashFunctionType.SimHash
    bucket_type: BucketType = BucketType.Fifo
    num_tables: int = 50
    range_pow: int = 6
    num_hashes: int = 6
    bucket_capacity: int = 128
    rebuild_interval_base: int = 100
    rebuild_decay: float = 0.1

    def to_c(self) -> _lib.LshConfigC:
        return _lib.LshConfigC(int(self.hash_function), int(self.bucket_type), self.num_tables, self.range_pow,
                               self.num_hashes, self.bucket_capacity, self.rebuild_interval_base,
                               float(self.rebuild_decay))


@dataclass
class LayerConfig:  # config.rs:67-106
    input_dim: int
    num_neurons: int
    activation: ActivationType = ActivationType.Relu
    lsh: LshConfig = field(default_factory=LshConfig)
    sampling: SamplingType = SamplingType.TopK
    sampling_threshold: int = 2
    top_k: int = 0
    is_output: bool = False

    @staticmethod
    def hidden(input_dim: int, num_neurons: int) -> "LayerConfig":  # config.rs:80-91
        return LayerConfig(input_dim, num_neurons, ActivationType.Relu, LshConfig(), SamplingType.TopK, 2,
                           num_neurons // 10, False)

    @staticmethod
    def output(input_dim: int, num_neurons: int) -> "LayerConfig":  # config.rs:93-104
        return LayerConfig(input_dim, num_neurons, ActivationType.Softmax, LshConfig(), SamplingType.TopK, 2,
                           num_neurons // 10, True)

    def to_c(self) -> _lib.LayerConfigC:
        return _lib.LayerConfigC(self.input_dim, self.num_neurons, int(self.activation), self.lsh.to_c(),
                                 int(self.sampling), self.sampling_threshold, self.top_k, int(self.is_output))


@dataclass
class NetworkConfig:  # config.rs:108-128
    layers: list = field(default_factory=list)
    optimizer: OptimizerType = OptimizerType.Adam
    learning_rate: float = 0.001
    batch_size: int = 128
    num_threads: int = 4


@dataclass
class SlideConfig:  # config.rs:130-143
    network: NetworkConfig = field(default_factory=NetworkConfig)
    seed: int = 42
    hogwild: bool = True

    def to_c(self, weight_dtype: int, max_batch: int):
        arr = (_lib.LayerConfigC * len(self.network.layers))(*[lc.to_c() for lc in self.network.layers])
        cfg = _lib.NetConfigC(len(self.network.layers), C.cast(arr, C.POINTER(_lib.LayerConfigC)),
                              int(self.network.optimizer), float(self.network.learning_rate),
                              self.network.batch_size, self.network.num_threads, self.seed, weight_dtype,
                              max_batch)
        return cfg, arr

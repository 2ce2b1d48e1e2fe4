"""B200 (sm_100a) CUDA backend for smallm-engine's batch-1 quantized decode.

Public surface (mirrors the reference's interfaces):
  CUDABackend   -- smallm::Backend (backend.h:12-38) on the GPU
  QMatrix       -- a device-resident repacked weight matrix
  CudaModel     -- smallm::Model (model.h:16-43): Qwen2/Llama decode on the GPU
  Generator     -- src/runtime/generator.cpp:22-72 over token ids
  synth         -- seeded synthetic GGUF models for the decode workloads
"""
from ._lib import SmallmError  # noqa: F401
from .backend import CUDABackend, QMatrix  # noqa: F401
from .model import (CudaModel, GenerationStats, Generator, GreedySampler, MT19937,  # noqa: F401
                    TemperatureSampler, TopKSampler, TopPSampler)

__all__ = ["SmallmError", "CUDABackend", "QMatrix", "CudaModel", "Generator", "GenerationStats",
           "TemperatureSampler", "TopKSampler", "TopPSampler",
           "GreedySampler", "MT19937"]

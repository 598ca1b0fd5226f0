"""qq3 -- B200 (sm_100a) backend for the QwenQwen3.js quantised inference path.

Layout:
  csrc/        CUDA kernels + the C ABI (include/qq3.h) -> libqq3cuda.so
  runtime.py   ctypes binding of the C ABI (what an N-API addon would wrap)
  engine.py    Qwen3CudaEngine / Lfm2CudaEngine: the reference engine API over the C ABI
  gguf.py      GGUF reader (the gguf.js API) and writer
  synth.py     seeded random-init Q8_0 models (libqq3synth.so)
  ep.py        expert-parallel LFM2-MoE block (torch.distributed exchange)
  tp.py        tensor-parallel dense Qwen3: shard plan, Q8_0 shards, the per-rank token step
  node/        N-API addon source + JS engine classes for a Node host
  build.py     in-tree build of the native libraries

The directory name is not a Python identifier, so loaders register it as ``qq3``.
"""
from . import build, ep, gguf, runtime, synth, tp  # noqa: F401
from .engine import Lfm2CudaEngine, Qwen3CudaEngine, engine_for  # noqa: F401

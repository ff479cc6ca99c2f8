"""eagle4_b200: a B200-native speculative-decoding framework with EAGLE-4 draft trees sized by a measured cost model.

Layers: ``core`` (cost model, draft tree, calibration; engine-free), ``models`` (targets and draft heads),
``ops`` (sm_100a kernels and their PyTorch oracles), ``parallel`` (tensor parallelism over NVLink), ``runtime``
(serving loop, caches, CUDA graphs), ``plugins`` (SGLang / vLLM / TokenSpeed entry points) and the CLI.
"""

__version__ = "0.1.0"

"""kvbm_b200: a Blackwell-native KV block manager.

Layers (bottom to top):

* ``kvbm_b200.ops``        - sm_100a CUDA kernels (libkvbm_cuda.so, C ABI)
* ``kvbm_b200.physical``   - pools, layouts, transfer planning and execution
* ``kvbm_b200.logical``    - block pool with sequence-hash prefix reuse (C++ core)
* ``kvbm_b200.engine``     - leader/worker engine, offload/onboard, sessions
* ``kvbm_b200.parallel``   - TP worker groups, P->D transfer over NVLink, collectives
* ``kvbm_b200.connector``  - vLLM KV-connector surface
* ``kvbm_b200.hub``        - coordination service (registry, indexer, prefill router)
* ``kvbm_b200.models``     - Llama-architecture driver harness
"""

__version__ = "0.1.0"

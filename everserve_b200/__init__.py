"""everserve_b200: a B200-native fault-tolerant LLM serving framework.

Layers (bottom to top): sm_100a kernels (``csrc/``, loaded by ``_ext``), decoder ops (``ops``),
models (``models``), the paged-KV continuous-batching engine (``engine``), the communication
runtime (``parallel``, ``runtime``), committed-KV state (``state``), the process <-> daemon contract
(``contract``), the CPU reference tier (``reference``), and the plugin surface (``plugin``). The
control plane (coordinator, node daemon, KV store) is C++ under ``cpp/``.
"""

__version__ = "0.1.0"

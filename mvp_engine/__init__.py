"""mvp_engine: a multimodal training engine for NVIDIA B200 (sm_100a).

Orchestration is PyTorch; the hot paths are hand-written sm_100a kernels
(``mvp_engine.ops``) and the data-parallel / context-parallel runtime lives in
``mvp_engine.parallel``.
"""

__version__ = "0.1.0"

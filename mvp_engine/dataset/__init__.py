"""Import-compatible name of the reference's (empty) ``mvp_engine.dataset`` package.

Datasets, sources and the streaming runtime of this engine live in :mod:`mvp_engine.data`; the data kits
(``mvp_engine.kit.llm.data``, ``mvp_engine.kit.mllm.data``) build on it."""
